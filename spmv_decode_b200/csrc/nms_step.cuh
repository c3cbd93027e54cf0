// Persistent decode step: every stage of one decode step (per layer: q/k/v
// GEMV, attention, o-projection, gate/up + SwiGLU, down-projection; then the
// output head with greedy argmax) runs inside ONE cooperative launch of one
// 640-thread CTA per SM (20 warps, 96 registers each; measured against 512,
// 576, 704 and 768 threads, this is the fastest: more warps hide more of the
// stage prologues' latency, fewer registers start to spill).
//
// Why: a batch-1 decode step is ~160 small HBM-bound launches.  Each launch
// pays a fixed cost (CTA start-up, the first loads' latency, the prologue,
// the tail) of several microseconds during which HBM idles.  Inside one
// persistent kernel the stages are separated by grid barriers instead, and
// every warp streams its weights through a shared-memory ring whose copies
// run ahead of the computation across stage boundaries (weights never
// depend on activations), so HBM keeps streaming while a CTA waits at a
// barrier, normalises its input or runs attention.
//
// Grid barrier: a monotonic arrival counter in global memory (reset by the
// last CTA to leave); waits are bounded by %globaltimer and record
// kDevBarrierTimeout instead of hanging.  Attention: one (KV head, context
// split) unit per CTA; the last unit of a head to finish (per-head arrival
// counter) combines the splits' partial softmax states from L2.
#pragma once

#include "nms_common.cuh"
#include "nms_decode.cuh"
#include "nms_gemv.cuh"

namespace nms {

#ifndef NMS_STEP_THREADS
#define NMS_STEP_THREADS 640
#endif
constexpr int kStepThreads = NMS_STEP_THREADS;
constexpr int kStepWarps = kStepThreads / kWarp;
constexpr uint64_t kBarrierLimitNs = 200ull * 1000 * 1000;
constexpr int kMaxSplits = 16;  // attention splits per KV head (cluster-size bound of the standalone kernel)

enum StageKind : int32_t { kStageGemv = 0, kStageAttn = 1 };
constexpr int kMaxTp = 8;
constexpr int kTraceMarks = 8;  // detail marks per stage and CTA

struct StepGemv;
struct ProdDesc;

struct StepParams {
  const int32_t* kind;      // [nstages] StageKind
  const StepGemv* gemv;     // [ngemv] GEMV stages in step order
  const ProdDesc* desc;     // [ngemv] their weight-stream descriptors
  const AttnParams* attn;   // [nattn] attention stages in step order
  int32_t nstages, ngemv, nattn;
  int32_t ring_bytes;       // kStepWarps * D * kRingItemBytes, at the start of dynamic shared memory
  int32_t act_bytes;        // working set after the rings (GEMV or attention); then desc[ngemv], kind[nstages]
  unsigned* bar_count;      // grid barrier arrivals (grows within a launch, reset at exit)
  unsigned* bar_exit;       // CTAs that have left the kernel (reset at exit)
  float* attn_part;         // [units][kAttnMaxGroup][kAttnD + 2] partial softmax states
  unsigned* attn_count;     // [Hkv] per-head arrival counters (return to 0)
  // Optional timeline (%globaltimer ns): trace[0] = kernel start (CTA 0);
  // trace[1 + s*(ncta+1) + c] = time CTA c finished stage s's work;
  // trace[1 + s*(ncta+1) + ncta] = time CTA 0 left the barrier after stage s.
  unsigned long long* trace;
  // Optional per-CTA detail after the timeline (SM clock cycles, clock64):
  // trace_detail[(s*ncta + c)*kTraceMarks + k], k = 0 stage entry; GEMV:
  // 1 input vector staged, 2 norm statistic done, 3 staged masks / norm
  // weights ready, 4 gathered vector built; attention: 4 first unit's q/k/v
  // prepared; then 5 main work done (GEMV: weight items consumed;
  // attention: partial state published), 6 stage finished.
  unsigned long long* trace_detail;
  const int64_t* pos;       // token position of the step (all attention stages)
  // Tensor parallelism (tp_world > 1): exchange areas of every rank as
  // mapped in this process (values[nreduce][world][dim] of {fp32, tag}),
  // this rank's own area, and the local count of completed steps.
  int32_t tp_world, tp_rank, tp_dim, tp_nreduce;
  uint2* tp_vals[kMaxTp];
  const uint2* tp_my_vals;
  unsigned long long* tp_epoch;
  // Vocabulary-parallel head (last stage, argmax): the local winner goes to
  // tp_local_best; the global token and the generation hooks are written here.
  int32_t tp_head, tp_vocab_offset;
  int64_t* tp_local_best;
  int64_t* tp_token_out;
  int64_t* tp_next_token;
  int64_t* tp_history;
  int64_t* tp_pos;
  int64_t tp_history_len;
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
// (kDevBarrierTimeout recorded) or found the device error word set.
__device__ __forceinline__ bool grid_wait(const unsigned* count, unsigned ncta, unsigned k) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = ncta * (k + 1);
    if (ld_acquire_u32(count) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_u32(count) < target) {
        // A recorded device error (a wait elsewhere gave up, or the host
        // asked for an abort) ends the wait at once: the step is void.
        if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) {
          ok = 0;
          break;
        }
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

// Called once by every CTA as it leaves, on the normal path and after an
// abandoned wait alike: the last one resets the barrier counter (no CTA of
// this launch reads it any more) and, under tensor parallelism, counts the
// step, so the next launch starts from zeroed counters and the exchange tags
// stay in step with the peers'.
__device__ __forceinline__ void step_exit(unsigned* count, unsigned* exit_count, unsigned ncta,
                                          unsigned long long* epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel_u32(exit_count, 1u);
    if (prev == ncta - 1) {
      atomicExch(count, 0u);
      atomicExch(exit_count, 0u);
      if (epoch != nullptr) atomicAdd(epoch, 1ull);  // steps completed (tensor-parallel exchange targets)
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange (one process per GPU, peers' areas mapped over
// NVLink).  Exchange point j of step e: every CTA of every rank writes each of
// its partial rows into slot [j][its rank] of every rank's area as ONE 8-byte
// store {fp32 value, tag}, tag = e * nreduce + j + 1 (never 0, the area
// starts zeroed).  An 8-byte store lands whole, so a reader that sees the
// expected tag sees the value: the data are their own arrival signal -- no
// fence, counter or cross-GPU barrier.  Readers (the next stage's prologue)
// poll each word they add.  Slots are reused one step later; a rank cannot
// reach step e + 1's point j before every rank has contributed to -- and so
// finished reading -- step e's points up to the last one.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t tp_tag(const StepParams& sp, unsigned long long epoch, int j) {
  return (uint32_t)(epoch * (unsigned long long)sp.tp_nreduce + (unsigned long long)j + 1ull);
}

__device__ __forceinline__ void tp_put(uint2* dst, float v, uint32_t tag) {
  asm volatile("st.relaxed.sys.global.v2.b32 [%0], {%1, %2};" ::"l"(dst), "r"(__float_as_uint(v)), "r"(tag)
               : "memory");
}

__device__ __forceinline__ uint2 tp_get(const uint2* src) {
  uint2 w;
  asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(src) : "memory");
  return w;
}

// Sum of exchange point j's partials for element i, in rank order (the same
// on every rank).  A word whose tag has not arrived is polled (bounded; after
// a recorded device error nobody waits any more).
__device__ __noinline__ uint2 tp_poll(const uint2* src, uint32_t tag) {
  uint2 w = tp_get(src);
  const uint64_t t0 = global_timer_ns();
  while (w.y != tag) {
    if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) break;
    if (global_timer_ns() - t0 > kBarrierLimitNs) {
      set_device_error(kDevBarrierTimeout);
      break;
    }
    w = tp_get(src);
  }
  return w;
}

__device__ __forceinline__ float tp_sum(const StepParams& sp, int j, int i, uint32_t tag) {
  const uint2* v = sp.tp_my_vals + (size_t)j * sp.tp_world * sp.tp_dim + i;
  float acc = 0.f;
  for (int r = 0; r < sp.tp_world; ++r) {
    uint2 w = tp_get(v + (size_t)r * sp.tp_dim);
    if (w.y != tag) w = tp_poll(v + (size_t)r * sp.tp_dim, tag);
    acc += __uint_as_float(w.x);
  }
  return acc;
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Weight streams.  Each warp owns a contiguous range of work items of every
// GEMV stage (an item: RG = 32/L rows x 16L halves, 32 bytes per lane) and
// streams them through its own shared-memory ring of D items with 16-byte
// cp.async copies (two per lane and item).  The producer side of the ring
// walks the warp's items of every GEMV stage of the step in order (a compact
// descriptor of every stage stays in shared memory), so the copies for the
// next stage are in flight while the CTA runs its epilogue, waits at the grid
// barrier, normalises the next input or runs attention -- weights never
// depend on activations.  Every consumed item commits exactly one copy group
// (empty past the step's last item), so `cp.async.wait_group D-1` always
// waits for exactly the item about to be read.  A lane only reads back the
// 32 bytes it copied itself.  Every active warp gets at least one row of
// items, so a row is split over at most two warps and its two shared-memory
// partial sums add in either order to the same value: results are
// deterministic.
// ---------------------------------------------------------------------------
constexpr int kRingItemBytes = kWarp * 32;
constexpr uint64_t kPreWaitLimitNs = 200ull * 1000 * 1000;

struct StepGemv {
  GemvParams g;
  int32_t lanes;    // L: lanes per row (32, 16, 8 or 4), w_pad % (16 L) == 0
  int32_t tp_send;  // tensor parallel: exchange point this stage's partial rows go to (-1: none)
  int32_t tp_recv;  // exchange point whose reduced vector is this stage's residual addend (-1: none)
  int32_t pad_;
};

// What the producer needs of a GEMV stage (64 bytes, all stages resident).
struct ProdDesc {
  const __half* w[kMaxSegs];
  int32_t row_start[kMaxSegs];
  int32_t rows_total, row_groups, w_pad;
  int16_t nseg;
  int8_t paired;
  int8_t lanes;
};
static_assert(sizeof(ProdDesc) == 64, "ProdDesc is 64 bytes");

__host__ __device__ inline int ring_lanes(int w_pad) {
  return (w_pad % 512 == 0) ? 32 : (w_pad % 256 == 0) ? 16 : (w_pad % 128 == 0) ? 8 : 4;
}

// A CTA's row groups [g0, g0 + ng) and a warp's items [t0, t1) of a stage.
struct WarpGeom {
  int cpr, g0, ng, t0, t1;
};

__device__ __forceinline__ WarpGeom warp_geom(int row_groups, bool paired, int w_pad, int L, unsigned cta,
                                              unsigned ncta, int warp) {
  WarpGeom q;
  q.cpr = w_pad / (16 * L);
  q.g0 = (int)(((unsigned)cta * (unsigned)row_groups) / ncta);
  q.ng = (int)(((unsigned)(cta + 1) * (unsigned)row_groups) / ncta) - q.g0;
  const int vgroups = paired ? 2 * q.ng : q.ng;
  const unsigned T = (unsigned)(vgroups * q.cpr);
  const int nw = max(1, min(kStepWarps, vgroups));  // >= cpr items per active warp
  if (warp < nw) {
    q.t0 = (int)(((unsigned)warp * T) / (unsigned)nw);
    q.t1 = (int)(((unsigned)(warp + 1) * T) / (unsigned)nw);
  } else {
    q.t0 = q.t1 = (int)T;
  }
  return q;
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Producer side of a warp's ring (lane-private registers; every lane runs it).
struct Prod {
  int n;          // GEMV ordinal whose items are being issued
  int t, t1;      // next item, end of this warp's items in that stage
  int vg, c, cpr; // row group, column item, items per row group
  int g0, ng;     // the CTA's row groups of the stage
  int cstep;      // bytes per column item (32 L)
  int slot;       // next ring slot
  const unsigned char* src;  // this lane's source at column item c of its row
  bool valid;
};

__device__ __forceinline__ void prod_row(Prod& P, const ProdDesc& d) {
  const int lane = threadIdx.x & 31, L = d.lanes, RG = kWarp / L;
  const int sub = lane / L, li = lane % L;
  int grow, segi = 0;
  if (d.paired) {
    segi = (P.vg >= P.ng) ? 1 : 0;
    grow = (P.g0 + P.vg - segi * P.ng) * RG + sub;
  } else {
    grow = (P.g0 + P.vg) * RG + sub;
#pragma unroll
    for (int k = 1; k < kMaxSegs; ++k)
      if (k < d.nseg && grow >= d.row_start[k]) segi = k;
  }
  P.valid = grow < d.rows_total;
  const int lrow = P.valid ? grow - (d.paired ? 0 : d.row_start[segi]) : 0;
  P.src = reinterpret_cast<const unsigned char*>(d.w[segi] + (size_t)lrow * d.w_pad) + li * 16 + P.c * P.cstep;
}

__device__ __forceinline__ void prod_setup(Prod& P, const ProdDesc& d, int n, unsigned cta, unsigned ncta) {
  const WarpGeom q = warp_geom(d.row_groups, d.paired != 0, d.w_pad, d.lanes, cta, ncta, threadIdx.x >> 5);
  P.n = n;
  P.t = q.t0;
  P.t1 = q.t1;
  P.cpr = q.cpr;
  P.g0 = q.g0;
  P.ng = q.ng;
  P.cstep = 32 * d.lanes;
  P.vg = q.t0 / q.cpr;
  P.c = q.t0 - P.vg * q.cpr;
  if (q.t0 < q.t1) prod_row(P, d);
}

// Commit one copy group: the warp's next item (moving on through the step's
// GEMV stages as needed), or an empty group past the last one.
template <int D>
__device__ __forceinline__ void prod_next(Prod& P, const ProdDesc* descs, int ngemv, unsigned char* wring,
                                          unsigned cta, unsigned ncta) {
  while (P.t >= P.t1 && P.n + 1 < ngemv) prod_setup(P, descs[P.n + 1], P.n + 1, cta, ncta);
  if (P.t < P.t1) {
    if (P.valid) {
      // Lane slots: first 16 bytes at +lane*16, second at +512 + lane*16
      // (conflict-free reads).
      unsigned char* dst = wring + P.slot * kRingItemBytes + (threadIdx.x & 31) * 16;
      cp_async_16(dst, P.src);
      cp_async_16(dst + 512, P.src + P.cstep / 2);
    }
    ++P.t;
    P.src += P.cstep;
    if (++P.c == P.cpr) {
      P.c = 0;
      ++P.vg;
      if (P.t < P.t1) prod_row(P, descs[P.n]);
    }
    P.slot = (P.slot + 1 == D) ? 0 : P.slot + 1;
  }
  cp_async_commit();
}

struct Ring {
  unsigned char* wring;  // this warp's D item slots
  int cslot;             // slot of the next item to consume
  Prod P;
};

// ---------------------------------------------------------------------------
// GEMV stage working set in shared memory (after the rings).
// ---------------------------------------------------------------------------
struct StepGemvSmem {
  __half* xs;     // [K] input after the residual add
  uint8_t* sidx;  // [nsegx][w_al] mask offsets
  __half* xc;     // [nsegx][w_pad] gathered input (natural order)
  __half* nw;     // [K] RMSNorm weight (norm prologue only)
  float* acc;     // [max_vrows] row sums
  float* red;     // [32] block reduction
};

__host__ __device__ inline size_t step_gemv_layout(int K, int w, int w_pad, int nsegx, int max_vrows, bool norm,
                                                   size_t* off_sidx, size_t* off_xc, size_t* off_nw, size_t* off_acc,
                                                   size_t* off_red) {
  size_t off = align_up_sz((size_t)K * 2, 16);
  *off_sidx = off;
  off += align_up_sz((size_t)w, 16) * nsegx;
  *off_xc = off;
  off += align_up_sz((size_t)w_pad * 2 * nsegx, 16);
  *off_nw = off;
  if (norm) off += align_up_sz((size_t)K * 2, 16);
  *off_acc = off;
  off += align_up_sz((size_t)max_vrows * 4, 16);
  *off_red = off;
  off += 32 * 4;
  return off;
}

__host__ __device__ inline size_t step_gemv_smem_bytes(int K, int w, int w_pad, int nsegx, int max_vrows, bool norm) {
  size_t a, b, c, d, e;
  return step_gemv_layout(K, w, w_pad, nsegx, max_vrows, norm, &a, &b, &c, &d, &e);
}

__device__ __forceinline__ StepGemvSmem step_gemv_smem(const GemvParams& p, unsigned char* base, int nsegx,
                                                       int max_vrows) {
  size_t o_sidx, o_xc, o_nw, o_acc, o_red;
  step_gemv_layout(p.K, p.w, p.w_pad, nsegx, max_vrows, p.prologue == kProResidNorm, &o_sidx, &o_xc, &o_nw, &o_acc,
                   &o_red);
  StepGemvSmem s;
  s.xs = reinterpret_cast<__half*>(base);
  s.sidx = base + o_sidx;
  s.xc = reinterpret_cast<__half*>(base + o_xc);
  s.nw = reinterpret_cast<__half*>(base + o_nw);
  s.acc = reinterpret_cast<float*>(base + o_acc);
  s.red = reinterpret_cast<float*>(base + o_red);
  return s;
}

__device__ __forceinline__ int stage_nsegx(const GemvParams& p) { return p.mode == kModePaired ? 2 : p.nseg; }
__device__ __forceinline__ int stage_max_vrows(const GemvParams& p, int RG, unsigned ncta) {
  return (p.mode == kModePaired ? 2 : 1) * ((p.row_groups + (int)ncta - 1) / (int)ncta) * RG;
}

// Mask offsets and RMSNorm weights of a GEMV stage: staged into the working
// set while the CTA waits at the grid barrier before the stage, by bulk
// copies (one thread issues; completion on an mbarrier, one phase per stage
// that uses it) when every piece is 16-byte shaped, else by plain loads.
__device__ __forceinline__ bool pre_bulk(const GemvParams& p) {
  if (p.seg[0].idx != nullptr) {
    if ((p.w & 15) != 0) return false;
    for (int sx = 0; sx < stage_nsegx(p); ++sx)
      if ((reinterpret_cast<uintptr_t>(p.seg[sx].idx) & 15u) != 0) return false;
  }
  if (p.prologue == kProResidNorm && ((p.K & 7) != 0 || (reinterpret_cast<uintptr_t>(p.norm_w) & 15u) != 0))
    return false;
  return true;
}

__device__ __forceinline__ void gemv_pre_smem(const StepGemv& sg, unsigned ncta, unsigned char* act, uint64_t* bar,
                                              unsigned& uses) {
  const GemvParams& p = sg.g;
  const int nsegx = stage_nsegx(p);
  StepGemvSmem s = step_gemv_smem(p, act, nsegx, stage_max_vrows(p, kWarp / sg.lanes, ncta));
  const int w_al = (int)align_up_sz((size_t)p.w, 16);
  const bool has_idx = p.seg[0].idx != nullptr, norm = p.prologue == kProResidNorm;
  if (pre_bulk(p)) {
    if (threadIdx.x == 0) {
      const uint32_t bytes = (has_idx ? (uint32_t)(nsegx * p.w) : 0u) + (norm ? (uint32_t)p.K * 2u : 0u);
      if (bytes > 0) {
        fence_proxy_async_smem();  // the CTA's earlier use of this memory (ordered by the block barrier) first
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
}

// One GEMV stage after its barrier: input prologue (residual add, RMSNorm
// statistic), gather, this warp's items from its ring (each consumed item
// commits the warp's next copy), epilogue.
// Stage the input vector (plus an addend, rounded to fp16 like the
// reference's residual add) into shared memory with 16-byte L2 reads, U per
// thread in flight at once; returns this thread's share of sum(x^2).
template <int U, bool ADD>
__device__ __forceinline__ float stage_input(const __half* x, const __half* x2, int K, __half* xs) {
  const int K8 = K >> 3;
  const uint4* xa = reinterpret_cast<const uint4*>(x);
  const uint4* xb = reinterpret_cast<const uint4*>(x2);
  float ss = 0.f;
  for (int base = threadIdx.x; base < K8; base += U * kStepThreads) {
    uint4 a[U], b[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i8 = base + u * kStepThreads;
      a[u] = b[u] = make_uint4(0u, 0u, 0u, 0u);
      if (i8 < K8) {
        a[u] = __ldcg(xa + i8);
        if (ADD) b[u] = __ldcg(xb + i8);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i8 = base + u * kStepThreads;
      if (i8 >= K8) break;
      const __half* ah = reinterpret_cast<const __half*>(&a[u]);
      const __half* bh = reinterpret_cast<const __half*>(&b[u]);
      uint4 o;
      __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __half hv = ADD ? f2h(h2f(ah[e]) + h2f(bh[e])) : ah[e];
        oh[e] = hv;
        ss = fmaf(h2f(hv), h2f(hv), ss);
      }
      *reinterpret_cast<uint4*>(xs + (size_t)i8 * 8) = o;
    }
  }
  return ss;
}

__device__ __forceinline__ void trace_at(unsigned long long* td, int k) {
  if (td != nullptr && threadIdx.x == 0) td[k] = clock64();
}

template <int L, int D>
__device__ __forceinline__ void gemv_stage(const StepParams& sp, const StepGemv& sg, const ProdDesc* descs, int ngemv,
                                           unsigned cta, unsigned ncta, unsigned char* act, Ring& R,
                                           uint64_t* pre_bar, unsigned pre_uses, unsigned long long epoch,
                                           unsigned long long* td) {
  constexpr int RG = kWarp / L, NT = kStepThreads, CB = 32 * L;
  const GemvParams& p = sg.g;
  const int tid = threadIdx.x, lane = tid & 31;
  const int sub = lane / L, li = lane % L;
  const WarpGeom q = warp_geom(p.row_groups, p.mode == kModePaired, p.w_pad, L, cta, ncta, tid >> 5);
  const bool paired = (p.mode == kModePaired);
  const int nsegx = stage_nsegx(p);
  const bool dense = (p.seg[0].idx == nullptr);
  const int max_vrows = stage_max_vrows(p, RG, ncta);
  StepGemvSmem s = step_gemv_smem(p, act, nsegx, max_vrows);
  const int w_al = (int)align_up_sz((size_t)p.w, 16);

  const __half* xsrc = input_row(p);
  const bool resid = (p.prologue == kProResidNorm);
  const bool add = resid && (p.x2 != nullptr);
  float ss = 0.f;
  if ((p.K & 7) == 0 && (reinterpret_cast<uintptr_t>(xsrc) & 15u) == 0 &&
      (!add || (reinterpret_cast<uintptr_t>(p.x2) & 15u) == 0)) {
    // The input (and residual addend) were written by other CTAs in the
    // previous stage: read them from L2, every load of a thread issued
    // before any is used (one round trip for K <= 32 * NT, or 16 * NT with
    // an addend).
    if (add)
      ss = stage_input<2, true>(xsrc, p.x2, p.K, s.xs);
    else
      ss = stage_input<4, false>(xsrc, nullptr, p.K, s.xs);
  } else {
    for (int i = tid; i < p.K; i += NT) {
      float v = h2f(xsrc[i]);
      if (add) v = h2f(f2h(v + h2f(p.x2[i])));
      s.xs[i] = f2h(v);
      ss = fmaf(v, v, ss);
    }
  }
  trace_at(td, 1);
  for (int v = tid; v < max_vrows; v += NT) s.acc[v] = 0.f;
  float rstd = 1.f;
  if (resid) {
    // (its first block barrier also publishes the staged input)
    const float tot = block_reduce_sum(ss, s.red);
    rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
  } else {
    __syncthreads();
  }
  trace_at(td, 2);
  if (resid && p.resid_out != nullptr && cta == 0)
    for (int i = tid; i < p.K; i += NT) p.resid_out[i] = s.xs[i];
  if (pre_bulk(p)) mbar_wait_bounded(pre_bar, (pre_uses - 1u) & 1u, kPreWaitLimitNs);  // staged masks / norm
  trace_at(td, 3);
  // Gather, four kept positions per thread and pass (one 4-byte read of
  // their mask offsets, one 8-byte store); consecutive threads take
  // consecutive positions, so their mask groups and shared-memory reads stay
  // together.  Offsets past w are never used (the staged rows are 16-byte
  // padded, so the 4-byte read stays inside them).
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
            if (resid) val = f2h(h2f(f2h(h2f(val) * rstd)) * h2f(s.nw[col]));
          }
        }
        v[e] = val;
      }
      *reinterpret_cast<uint2*>(xc + j0) = *reinterpret_cast<const uint2*>(v);
    }
  }
  __syncthreads();
  trace_at(td, 4);

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
  if (sg.tp_send >= 0) {
    // Row-parallel shard: this CTA's fp32 partial rows go to slot
    // [tp_send][rank] of every rank's exchange area (over NVLink).
    const int row_lo = q.g0 * RG;
    const int nrows = min(q.ng * RG, max(0, p.rows_total - row_lo));
    const size_t off = ((size_t)sg.tp_send * sp.tp_world + sp.tp_rank) * sp.tp_dim + row_lo;
    const uint32_t stag = tp_tag(sp, epoch, sg.tp_send);
    for (int k = tid; k < nrows * sp.tp_world; k += NT) {
      const int r = k / nrows, v = k - r * nrows;
      tp_put(sp.tp_vals[r] + off + v, s.acc[v], stag);
    }
  } else {
    gemv_epilogue<NT>(p, s.acc, q.g0, q.ng, RG, cta, ncta);
  }
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

__device__ __forceinline__ void attention_unit(const AttnParams& p, int pos_in, int split, int kvh, StepAttnSmem& S,
                                               float* part, unsigned* head_count, unsigned long long* td) {
  constexpr int D = kAttnD, PT = kAttnTile, GM = kAttnMaxGroup, NT = kStepThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  if (pos_in < 0 || pos_in >= p.S_max) {  // uniform: every CTA read the same value
    if (tid == 0 && split == 0 && kvh == 0) set_device_error(kDevBadPosition);
    return;
  }
  const int pos = pos_in;
  const int P = pos + 1;
  const int pb = (int)(((int64_t)split * P) / p.splits);
  const int pe = (int)(((int64_t)(split + 1) * P) / p.splits);
  const bool has_new = (split == p.splits - 1);
  const __half* rope_row = p.rope + (size_t)pos * D;
  const __half* kbase = p.k_cache + (size_t)kvh * p.S_max * D;
  const __half* vbase = p.v_cache + (size_t)kvh * p.S_max * D;
  // K and V rows of a tile: cached rows by plain 16-byte loads into
  // registers (kept apart from the weight streams' copy groups), stored to
  // shared memory once the q / k / v work is done; rows past the range are
  // zero; the new token's row is filled from shared memory later.  Rows
  // before `pos` are never written during the step, so they are read through
  // the non-coherent path.
  constexpr int PIECES = 2 * PT * (D / 8);
  constexpr int PPT = (PIECES + NT - 1) / NT;  // pieces per thread
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
  if (pb < pe) load_tile(pb);  // in flight during the q / k / v work below

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
  trace_at(td, 4);

  for (int t0 = pb; t0 < pe; t0 += PT) {
    const int nt = min(PT, pe - t0);
    if (t0 != pb) load_tile(t0);
    store_tile(t0);
    __syncthreads();  // knew / vnew (written above) visible
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

  // Publish this split's state [g][m, l, o[D]] and count arrivals per head.
  constexpr int STRIDE = D + 2;
  float* my = part + ((size_t)kvh * p.splits + split) * GM * STRIDE;
  for (int i = tid; i < G * STRIDE; i += NT) {
    const int g = i / STRIDE, k = i - g * STRIDE;
    my[g * STRIDE + k] = (k == 0) ? S.sm[g] : (k == 1) ? S.sl[g] : S.so[g][k - 2];
  }
  __syncthreads();
  if (tid == 0) {
    // One acquire-release add: it publishes this CTA's partial state (the
    // block barrier above makes the other threads' stores part of it) and,
    // for the last unit of the head, makes every other unit's state visible
    // -- cheaper than a sequentially consistent fence on each side.
    const unsigned prev = atom_add_acq_rel_u32(&head_count[kvh], 1u);
    S.last = (prev == (unsigned)p.splits - 1) ? 1 : 0;
    if (S.last) head_count[kvh] = 0u;
  }
  __syncthreads();
  trace_at(td, 5);
  if (!S.last) return;
  // Last split of this head: combine every split's state, read through L2.
  // The partial outputs a thread weights are loaded together with the
  // (m, l) pairs (one round trip), and the split weights of a query head are
  // computed by one lane per split with shuffles.
  const float* hp = part + (size_t)kvh * p.splits * GM * STRIDE;
  float* fw = &S.so[0][0];   // per (split, head) weight exp(m_r - M) / L
  constexpr int IPT = (kAttnMaxGroup * D + NT - 1) / NT;  // output items per thread
  float ov[IPT][kMaxSplits];
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const int i = tid + k * NT;
    const int g = i / D, d = i - g * D;
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r)
      ov[k][r] = (i < G * D && r < p.splits) ? __ldcg(hp + ((size_t)r * GM + g) * STRIDE + 2 + d) : 0.f;
  }
  const bool fast = (p.splits & (p.splits - 1)) == 0 && p.splits <= kWarp && G * p.splits <= NT;
  if (fast) {
    // Lane group of `splits` lanes per query head: i = g * splits + r.
    const int i = tid, g = i / p.splits, r = i - g * p.splits;
    const bool on = i < G * p.splits;
    const float mr = on ? __ldcg(hp + ((size_t)r * GM + g) * STRIDE) : -INFINITY;
    const float lr = on ? __ldcg(hp + ((size_t)r * GM + g) * STRIDE + 1) : 0.f;
    float M = mr;
    for (int o = p.splits >> 1; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float f = (mr == -INFINITY) ? 0.f : expf(mr - M);
    float Ls = lr * f;
    for (int o = p.splits >> 1; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
    if (on) fw[r * GM + g] = f / Ls;
  } else {
    float* mlr = &S.sq[0][0];  // per (split, head) (m, l)
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
  }
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
      p.y[(size_t)(kvh * G + g) * D + d] = f2h(O);
    }
  }
}

// Vocabulary-parallel greedy token (one thread, after this GPU's head stage):
// the rank's (logit, global index) candidate goes to point `nreduce` of every
// rank's area; the largest logit wins, the lowest index on ties -- the token
// argmax over the full logits gives.  Then the head's generation hooks.
__device__ __forceinline__ void tp_head_token(const StepParams& sp, const GemvParams& hp, unsigned long long epoch) {
  const __half* logits = hp.out;
  const int64_t li = *reinterpret_cast<volatile int64_t*>(sp.tp_local_best);
  // The rank's candidate value: its winner's fp16 logit, or (temperature
  // sampling) the same key the local argmax compared.
  float lv = h2f(logits[li]);
  if (hp.temperature > 0.f)
    lv = lv * (1.0f / hp.temperature) +
         gumbel_noise(hp.sample_seed, hp.sample_pos != nullptr ? *hp.sample_pos : 0, li + hp.sample_row_offset);
  const uint32_t tag = tp_tag(sp, epoch, sp.tp_nreduce);
  const size_t slot = ((size_t)sp.tp_nreduce * sp.tp_world + sp.tp_rank) * sp.tp_dim;
  for (int r = 0; r < sp.tp_world; ++r) {
    tp_put(sp.tp_vals[r] + slot, lv, tag);
    tp_put(sp.tp_vals[r] + slot + 1, __uint_as_float((uint32_t)(li + sp.tp_vocab_offset)), tag);
  }
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int r = 0; r < sp.tp_world; ++r) {
    const uint2* c = sp.tp_my_vals + ((size_t)sp.tp_nreduce * sp.tp_world + r) * sp.tp_dim;
    uint2 wv = tp_get(c), wi = tp_get(c + 1);
    if (wv.y != tag) wv = tp_poll(c, tag);
    if (wi.y != tag) wi = tp_poll(c + 1, tag);
    const float v = __uint_as_float(wv.x);
    if (v > bv || (v == bv && wi.x < bi)) {
      bv = v;
      bi = wi.x;
    }
  }
  const int64_t tok = (int64_t)bi;
  *sp.tp_token_out = tok;
  if (sp.tp_next_token != nullptr) *sp.tp_next_token = tok;
  if (sp.tp_pos != nullptr) {
    const int64_t cur = *sp.tp_pos;
    if (sp.tp_history != nullptr && cur >= 0 && cur < sp.tp_history_len) sp.tp_history[cur] = tok;
    *sp.tp_pos = cur + 1;
  }
}

// ---------------------------------------------------------------------------
// L2 residency of the step's small constant operands (mask offsets, RMSNorm
// weights).  The weight rings keep tens of MB of requests queued in HBM, so
// an operand that has to come from HBM at a stage boundary waits behind
// them; with an evict-last prefetch at the start of every step these
// operands stay in L2 while the weight stream (evict-normal) passes through.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_l2_evict_last(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

__device__ __forceinline__ void pin_small_operands(const StepParams& sp, unsigned cta, unsigned ncta) {
  for (int gi = (int)cta; gi < sp.ngemv; gi += (int)ncta) {
    const GemvParams& p = sp.gemv[gi].g;
    const int nsegx = p.mode == kModePaired ? 2 : p.nseg;
    int k = threadIdx.x;
    if (p.seg[0].idx != nullptr) {
      for (int sx = 0; sx < nsegx; ++sx) {
        const int lines = (p.w + 127) >> 7;
        for (; k < lines; k += kStepThreads) prefetch_l2_evict_last(p.seg[sx].idx + ((size_t)k << 7));
        k -= lines;
      }
    }
    if (p.prologue == kProResidNorm && p.norm_w != nullptr) {
      const int lines = (p.K * 2 + 127) >> 7;
      for (; k < lines; k += kStepThreads)
        prefetch_l2_evict_last(reinterpret_cast<const char*>(p.norm_w) + ((size_t)k << 7));
    }
  }
}

// K/V rows [0, pos] of an attention stage pulled into L2 while the stage
// before it runs (the attention's first loads are then L2 hits instead of
// waiting behind the weight stream's queued requests).
__device__ __forceinline__ void prefetch_kv_l2(const AttnParams& a, int pos, unsigned cta, unsigned ncta) {
  if (threadIdx.x != 0 || pos < 0 || pos >= a.S_max) return;
  constexpr uint32_t kChunk = 16384;
  const uint32_t bytes = (uint32_t)(pos + 1) * kAttnD * 2;
  const uint32_t per = (bytes + kChunk - 1) / kChunk;
  const uint32_t total = 2u * (uint32_t)a.Hkv * per;
  for (uint32_t c = cta; c < total; c += ncta) {
    const uint32_t which = c / ((uint32_t)a.Hkv * per), rem = c - which * (uint32_t)a.Hkv * per;
    const uint32_t h = rem / per, q = rem - h * per;
    const char* base = reinterpret_cast<const char*>((which ? a.v_cache : a.k_cache) + (size_t)h * a.S_max * kAttnD);
    const uint32_t off = q * kChunk, n = min(kChunk, bytes - off);
    bulk_prefetch_l2(base + off, n);
  }
}

// ---------------------------------------------------------------------------
// The persistent kernel (D: ring depth in items per warp).
// ---------------------------------------------------------------------------
constexpr int kGemvWords = (int)(sizeof(StepGemv) / 4);
constexpr int kAttnWords = (int)(sizeof(AttnParams) / 4);
static_assert(sizeof(StepGemv) % 4 == 0 && sizeof(AttnParams) % 4 == 0, "parameter blocks are copied as words");
static_assert(kGemvWords <= kStepThreads && kAttnWords <= kStepThreads, "one parameter word per thread");

template <int D>
__device__ __forceinline__ void run_gemv(const StepParams& sp, const StepGemv& sg, const ProdDesc* descs, int ngemv,
                                         unsigned cta, unsigned ncta, unsigned char* act, Ring& R, uint64_t* pre_bar,
                                         unsigned pre_uses, unsigned long long epoch, unsigned long long* td) {
  switch (sg.lanes) {
    case 32: gemv_stage<32, D>(sp, sg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, epoch, td); break;
    case 16: gemv_stage<16, D>(sp, sg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, epoch, td); break;
    case 8: gemv_stage<8, D>(sp, sg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, epoch, td); break;
    default: gemv_stage<4, D>(sp, sg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, epoch, td); break;
  }
}

template <int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams sp) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ StepGemv s_g[2];        // GEMV parameters by ordinal parity
  __shared__ AttnParams s_attn[2];   // attention parameters by ordinal parity
  __shared__ int s_pos;
  __shared__ uint64_t s_pre_bar;     // staging of a stage's masks / norm weights
  const unsigned cta = blockIdx.x, ncta = gridDim.x;
  const int tid = threadIdx.x;
  unsigned char* act = smem_raw + sp.ring_bytes;
  ProdDesc* s_desc = reinterpret_cast<ProdDesc*>(act + sp.act_bytes);  // [ngemv]
  int* s_kind = reinterpret_cast<int*>(s_desc + sp.ngemv);               // [nstages]

  for (int s = tid; s < sp.nstages; s += kStepThreads) s_kind[s] = sp.kind[s];
  for (int i = tid; i < sp.ngemv * (int)(sizeof(ProdDesc) / 16); i += kStepThreads)
    reinterpret_cast<uint4*>(s_desc)[i] = __ldg(reinterpret_cast<const uint4*>(sp.desc) + i);
  if (tid < kGemvWords && sp.ngemv > 0)
    reinterpret_cast<uint32_t*>(&s_g[0])[tid] = reinterpret_cast<const uint32_t*>(sp.gemv)[tid];
  if (tid < kAttnWords && sp.nattn > 0)
    reinterpret_cast<uint32_t*>(&s_attn[0])[tid] = reinterpret_cast<const uint32_t*>(sp.attn)[tid];
  if (tid == 0) mbar_init(&s_pre_bar, 1);
  unsigned pre_uses = 0;  // phases of s_pre_bar started (uniform)
  __syncthreads();
  // Weights are constant: fill every warp's ring before waiting for the
  // predecessor grid.
  Ring R;
  R.wring = smem_raw + (size_t)(tid >> 5) * D * kRingItemBytes;
  R.cslot = 0;
  R.P.n = -1;
  R.P.t = R.P.t1 = 0;
  R.P.slot = 0;
  for (int i = 0; i < D; ++i) prod_next<D>(R.P, s_desc, sp.ngemv, R.wring, cta, ncta);

  grid_dep_wait();
  if (sp.trace != nullptr && cta == 0 && tid == 0) sp.trace[0] = global_timer_ns();
#if NMS_STEP_PF_SMALL
  pin_small_operands(sp, cta, ncta);
#endif
  // The token position is fixed for the whole step (the head advances it as
  // the last thing the step does): read it once.
  if (tid == 0) s_pos = (sp.pos != nullptr) ? (int)min((int64_t)0x7fffffff, max((int64_t)-1, *sp.pos)) : 0;
  if (sp.nstages > 0 && s_kind[0] == kStageGemv) gemv_pre_smem(s_g[0], ncta, act, &s_pre_bar, pre_uses);
  __syncthreads();
  int gn = 0, an = 0;  // ordinals of the next GEMV / attention stage
  bool aborted = false;  // a grid barrier wait was abandoned (uniform per CTA)
  const unsigned long long epoch = (sp.tp_world > 1) ? *reinterpret_cast<volatile unsigned long long*>(sp.tp_epoch) : 0ull;
  for (int s = 0; s < sp.nstages; ++s) {
    int tp_j = -1;            // exchange point this stage feeds (tensor parallel)
    __half* tp_out = nullptr;
    unsigned long long* td = sp.trace_detail ? sp.trace_detail + ((size_t)s * ncta + cta) * kTraceMarks : nullptr;
    trace_at(td, 0);
#if NMS_STEP_PF_KV
    if (s + 1 < sp.nstages && s_kind[s + 1] == kStageAttn) prefetch_kv_l2(s_attn[an & 1], s_pos, cta, ncta);
#endif
    if (s_kind[s] == kStageGemv) {
      // The next GEMV stage's parameters: loaded now, stored after this
      // stage into the slot GEMV gn-1 used.
      const bool more = gn + 1 < sp.ngemv;
      uint32_t stash = 0u;
      if (more && tid < kGemvWords) stash = __ldg(reinterpret_cast<const uint32_t*>(sp.gemv + gn + 1) + tid);
      tp_j = s_g[gn & 1].tp_send;
      tp_out = s_g[gn & 1].g.out;
      run_gemv<D>(sp, s_g[gn & 1], s_desc, sp.ngemv, cta, ncta, act, R, &s_pre_bar, pre_uses, epoch, td);
      if (more && tid < kGemvWords) reinterpret_cast<uint32_t*>(&s_g[(gn + 1) & 1])[tid] = stash;
      ++gn;
    } else {
      const bool more = an + 1 < sp.nattn;
      uint32_t stash = 0u;
      if (more && tid < kAttnWords) stash = __ldg(reinterpret_cast<const uint32_t*>(sp.attn + an + 1) + tid);
      const AttnParams& a = s_attn[an & 1];
      const int units = a.Hkv * a.splits;
      StepAttnSmem& A = *reinterpret_cast<StepAttnSmem*>(act);
      for (int u = cta; u < units; u += ncta) {
        attention_unit(a, s_pos, u % a.splits, u / a.splits, A, sp.attn_part, sp.attn_count, u == (int)cta ? td : nullptr);
        __syncthreads();
      }
      if (more && tid < kAttnWords) reinterpret_cast<uint32_t*>(&s_attn[(an + 1) & 1])[tid] = stash;
      ++an;
    }
    unsigned long long* tr = sp.trace ? sp.trace + 1 + (size_t)s * (ncta + 1) : nullptr;
    if (tr != nullptr && tid == 0) tr[cta] = global_timer_ns();
    trace_at(td, 6);
    if (tp_j >= 0) {
      // Tensor-parallel exchange point: the partial rows went out in the
      // epilogue carrying their arrival tags.  Each CTA sums its slice of the
      // vector over the ranks (rank order) into the stage's own output, then
      // the usual grid barrier: the next stage reads the reduced vector as
      // its residual addend, like the single-GPU step.
      {
        const uint32_t tag = tp_tag(sp, epoch, tp_j);
        const int i0 = (int)(((int64_t)cta * sp.tp_dim) / ncta), i1 = (int)(((int64_t)(cta + 1) * sp.tp_dim) / ncta);
        for (int i = i0 + tid; i < i1; i += kStepThreads) tp_out[i] = f2h(tp_sum(sp, tp_j, i, tag));
      }
      if (s + 1 < sp.nstages) {
        grid_arrive(sp.bar_count);
        if (s_kind[s + 1] == kStageGemv) gemv_pre_smem(s_g[gn & 1], ncta, act, &s_pre_bar, pre_uses);
        if (!grid_wait(sp.bar_count, ncta, (unsigned)s)) {
          aborted = true;
          break;
        }
      }
      if (tr != nullptr && cta == 0 && tid == 0) tr[ncta] = global_timer_ns();
    } else if (s + 1 < sp.nstages) {
      grid_arrive(sp.bar_count);  // includes __syncthreads: the stored parameters are visible
      if (s_kind[s + 1] == kStageGemv) gemv_pre_smem(s_g[gn & 1], ncta, act, &s_pre_bar, pre_uses);
      if (!grid_wait(sp.bar_count, ncta, (unsigned)s)) {
        aborted = true;
        break;
      }
      if (tr != nullptr && cta == 0 && tid == 0) tr[ncta] = global_timer_ns();
    }
  }
  if (aborted) {
    // An abandoned wait: the staging of the next stage's masks / norm
    // weights started before it may still be in flight; no copy may land
    // after exit.  Then leave through step_exit like every other CTA.
    if (tid == 0 && pre_uses > 0u) mbar_wait_bounded(&s_pre_bar, (pre_uses - 1u) & 1u, kPreWaitLimitNs);
    __syncthreads();
  } else if (sp.tp_world > 1 && sp.tp_head) {
    // The head's last CTA wrote this rank's winner; every CTA has written its
    // logits: one grid barrier, then CTA 0 swaps candidates with the peers.
    grid_arrive(sp.bar_count);
    if (grid_wait(sp.bar_count, ncta, (unsigned)sp.nstages - 1u) && cta == 0 && tid == 0)
      tp_head_token(sp, s_g[(gn - 1) & 1].g, epoch);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  step_exit(sp.bar_count, sp.bar_exit, ncta, sp.tp_world > 1 ? sp.tp_epoch : nullptr);
  grid_dep_launch_dependents();
}

// Ring depths the persistent kernel is built for (the host takes the largest
// whose rings fit next to the step's working set).
#ifndef NMS_STEP_DEPTH_HI
#define NMS_STEP_DEPTH_HI 8
#define NMS_STEP_DEPTH_LO 4
#endif
constexpr int kStepDepthHi = NMS_STEP_DEPTH_HI;
constexpr int kStepDepthLo = NMS_STEP_DEPTH_LO;

}  // namespace nms
