// Shared-mask N:M sparse GEMV kernels for batch-1 decode on sm_100a.
//
// Semantics (reference: triton_spmv.py:81-108, the nmsparse kernels' hot
// loop):  out[r] = sum_g sum_i  W[g*n + i, r] * x[g*m + idx[g, i]]
// with W the kept fp16 values, idx the uint8 in-group offsets shared by every
// output row, and fp32 fused multiply-add accumulation.
//
// Because the mask is shared by all rows, the gathered vector
//     xc[j] = x[(j / n) * m + idx[j]],   j in [0, w),  w = K*n/m
// is the same for every row: each CTA builds it once in shared memory, and
// the rest is a dense GEMV over the compressed width that streams the
// weights from HBM with 256-bit evict-first loads.
//
// Two weight layouts:
//   * reference layout  mat_data[w, h]  (element (j, r) at j*h + r) -- the
//     layout the reference packer produces and `nmsparse::gemv` accepts.
//   * packed layout     packed[h, w_pad] (row r contiguous, zero padded to
//     w_pad) -- produced by nms_pack_f16; each CTA owns whole output rows,
//     so no cross-CTA reduction, no atomics to global memory, no memset.
#pragma once

#include "nms_common.cuh"

namespace nms {

constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / kWarp;
constexpr int kMaxSegs = 4;

enum GemvMode : int32_t {
  kModeConcat = 0,  // segments' rows are concatenated in the output (fused q/k/v)
  kModePaired = 1,  // two segments with equal rows; out[r] = silu(seg0[r]) * seg1[r]
};
enum GemvPrologue : int32_t {
  kProPlain = 0,      // xin = x
  kProResidNorm = 1,  // xin = fp16(x + x2) (x2 optional); x fed to GEMV = rmsnorm(xin) * norm_w
};
enum GemvEpilogue : int32_t {
  kEpiStore = 0,   // out[r] = fp16(acc)
  kEpiSwiGLU = 1,  // paired mode only
  kEpiArgmax = 2,  // out[r] = fp16(acc) (logits) and argmax over all rows -> token_out
};

struct GemvSeg {
  const __half* w;     // packed [rows, w_pad]
  const uint8_t* idx;  // [w/n, n] shared-mask offsets; nullptr = dense row (w == K)
  int32_t rows;
  int32_t row_start;  // concat mode: first output row of this segment
};

struct GemvParams {
  GemvSeg seg[kMaxSegs];
  int32_t nseg;
  int32_t mode;
  int32_t prologue;
  int32_t epilogue;
  int32_t K;      // input features
  int32_t n, m;   // kept per group, group width (ignored for dense segments)
  int32_t w;      // compressed width
  int32_t w_pad;  // packed row stride, multiple of 16*L
  int32_t rows_total;  // concat: sum of segment rows; paired: rows of each segment
  int32_t row_groups;  // ceil(rows_total / RG)
  int32_t pf_items;        // per-warp L2 look-ahead (work items of 1 KB) ahead of the register ring
  const char* next_pf[2];  // weights of the next launch (see prefetch_shares_l2)
  uint32_t next_pf_bytes[2];
  uint32_t next_pf_head;
  const __half* x;          // input vector, or a [x_rows, K] table when x_token is set
  const int64_t* x_token;   // optional: the input is row *x_token of the table x (embedding)
  int64_t x_rows;
  const __half* x2;
  const __half* norm_w;
  float eps;
  __half* resid_out;
  __half* out;
  float* amax_val;       // [gridDim.x] argmax partials
  int32_t* amax_idx;     // [gridDim.x]
  uint32_t* amax_counter;  // zero before the first launch; reset by the last CTA
  int64_t* token_out;
  // Generation hooks of the argmax epilogue (each optional):
  int64_t* next_token;     // also write the token here (next step's input id)
  int64_t* token_history;  // history[*pos] = token
  int64_t* pos;            // position counter, incremented after the above
  int64_t history_len;     // entries in token_history
  // Temperature sampling in the argmax epilogue (temperature > 0): the token
  // is argmax(logit / temperature + Gumbel noise(seed, *sample_pos, row +
  // sample_row_offset)) -- a sample of softmax(logit / temperature).
  float temperature;       // 0: greedy argmax
  int32_t pad_s;
  uint64_t sample_seed;
  const int64_t* sample_pos;  // noise counter (the token position), or nullptr (0)
  int64_t sample_row_offset;  // global vocabulary row of local row 0 (vocabulary-parallel head)
};

// Position of compressed element j inside the permuted shared-memory copy of
// xc.  A chunk is the 16*L halves that L lanes read with one 32-byte load
// each; lane u's 16 values are split into two 8-value halves stored at
// u*8 and L*8 + u*8, so that each of the two 16-byte shared loads of a warp
// touches consecutive addresses (conflict-free).
template <int L>
__device__ __forceinline__ int xc_perm(int j) {
  const int c = j / (16 * L);
  const int o = j - c * (16 * L);
  const int u = o >> 4;
  const int e = o & 15;
  return c * (16 * L) + (e >> 3) * (8 * L) + u * 8 + (e & 7);
}

struct GemvSmem {
  __half* xs;     // [K] staged input (after residual add)
  uint8_t* sidx;  // [nsegx][w_al] staged mask offsets
  __half* xc;     // [nsegx][w_pad] permuted gathered vectors
  float* acc;     // [virtual rows of this CTA]
  float* red;     // [32]
  uint64_t* bar;  // [2] mbarriers: 0 = mask offsets, 1 = x
};

__host__ __device__ inline size_t align_up_sz(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared memory layout (host and device agree on it).
__host__ __device__ inline size_t gemv_smem_bytes(int K, int w, int w_pad, int nsegx, int max_vrows) {
  size_t off = align_up_sz((size_t)K * 2, 16);
  off += align_up_sz((size_t)w, 16) * nsegx;
  off += align_up_sz((size_t)w_pad * 2 * nsegx, 16);
  off += align_up_sz((size_t)max_vrows * 4, 16);
  off += 32 * 4;
  off += 16;
  return off;
}

// The GEMV input vector: p.x, or row *p.x_token of the table p.x (the token
// embedding folded into the first GEMV of a decode step).  Must be called
// after the dependency wait (the token is produced by the previous step).
__device__ __forceinline__ const __half* input_row(const GemvParams& p) {
  if (p.x_token == nullptr) return p.x;
  int64_t t = *p.x_token;
  if (t < 0 || t >= p.x_rows) t = 0;  // host validates the ids it supplies
  return p.x + (size_t)t * p.K;
}

// Row owned by this lane's subgroup for virtual row-group `vg` of the CTA.
struct LaneRow {
  int segi;   // segment
  int lrow;   // row inside the segment
  bool valid;
};

__device__ __forceinline__ LaneRow lane_row(const GemvParams& p, bool paired, int g0, int ng, int vg, int RG,
                                            int sub) {
  LaneRow r;
  if (paired) {
    r.segi = (vg >= ng) ? 1 : 0;
    const int grow = (g0 + vg - r.segi * ng) * RG + sub;
    r.valid = grow < p.rows_total;
    r.lrow = r.valid ? grow : 0;
  } else {
    const int grow = (g0 + vg) * RG + sub;
    r.valid = grow < p.rows_total;
    r.segi = 0;
#pragma unroll
    for (int q = 1; q < kMaxSegs; ++q)
      if (q < p.nseg && grow >= p.seg[q].row_start) r.segi = q;
    r.lrow = r.valid ? grow - p.seg[r.segi].row_start : 0;
  }
  return r;
}

// Epilogue over a CTA's rows [g0*RG, g0*RG + ng*RG): store, SwiGLU or
// store + grid-wide argmax (last CTA reduces the per-CTA partials).
template <int NT>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, const float* acc, int g0, int ng, int RG,
                                              unsigned cta, unsigned ncta) {
  constexpr int NWE = NT / kWarp;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* s_acc = acc;
  const int row_lo = g0 * RG;
  const int nrows = min(ng * RG, max(0, p.rows_total - row_lo));
  if (p.epilogue == kEpiSwiGLU) {
    for (int v = tid; v < nrows; v += NT) {
      const float g = h2f(f2h(s_acc[v]));
      const float u = h2f(f2h(s_acc[ng * RG + v]));
      const float sg = h2f(f2h(g / (1.0f + expf(-g))));
      p.out[row_lo + v] = f2h(sg * u);
    }
  } else if (p.epilogue == kEpiStore) {
    for (int v = tid; v < nrows; v += NT) p.out[row_lo + v] = f2h(s_acc[v]);
  } else {  // argmax
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const bool sample = p.temperature > 0.f;
    const float inv_t = sample ? 1.0f / p.temperature : 1.f;
    const int64_t spos = (sample && p.sample_pos != nullptr) ? *p.sample_pos : 0;
    for (int v = tid; v < nrows; v += NT) {
      const __half hv = f2h(s_acc[v]);
      p.out[row_lo + v] = hv;
      const int row = row_lo + v;
      // The fp16 logit (greedy), or its sampling key.
      const float fv = sample ? h2f(hv) * inv_t + gumbel_noise(p.sample_seed, spos, row + p.sample_row_offset)
                              : h2f(hv);
      if (fv > bv || (fv == bv && row < bi)) {
        bv = fv;
        bi = row;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    __shared__ float sv[NWE];
    __shared__ int si[NWE];
    __shared__ int s_last;
    if (lane == 0) {
      sv[warp] = bv;
      si[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int q = 1; q < NWE; ++q) {
        if (sv[q] > bv || (sv[q] == bv && si[q] < bi)) {
          bv = sv[q];
          bi = si[q];
        }
      }
      p.amax_val[cta] = bv;
      p.amax_idx[cta] = bi;
      const uint32_t prev = atom_add_acq_rel_u32(p.amax_counter, 1u);
      s_last = (prev == ncta - 1) ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      // Last CTA to finish: reduce all partials (each CTA wrote its partial
      // before its acquire-release counter add, so they are visible here).
      float fv = -INFINITY;
      int fi = 0x7fffffff;
      for (int q = tid; q < (int)ncta; q += NT) {
        const float qv = __ldcg(p.amax_val + q);
        const int qi = __ldcg(p.amax_idx + q);
        if (qv > fv || (qv == fv && qi < fi)) {
          fv = qv;
          fi = qi;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, fv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, fi, o);
        if (ov > fv || (ov == fv && oi < fi)) {
          fv = ov;
          fi = oi;
        }
      }
      __syncthreads();
      if (lane == 0) {
        sv[warp] = fv;
        si[warp] = fi;
      }
      __syncthreads();
      if (tid == 0) {
        for (int q = 1; q < NWE; ++q) {
          if (sv[q] > fv || (sv[q] == fv && si[q] < fi)) {
            fv = sv[q];
            fi = si[q];
          }
        }
        *p.token_out = (int64_t)fi;
        if (p.next_token != nullptr) *p.next_token = (int64_t)fi;
        if (p.pos != nullptr) {
          const int64_t cur = *p.pos;
          if (p.token_history != nullptr && cur >= 0 && cur < p.history_len) p.token_history[cur] = (int64_t)fi;
          *p.pos = cur + 1;
        }
        *p.amax_counter = 0u;
      }
    }
  }
}

template <int L>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_packed_kernel(const __grid_constant__ GemvParams p) {
  constexpr int RG = kWarp / L;  // rows processed together by one warp
  constexpr int U = 4;           // depth of the per-lane register ring (32-byte loads in flight)
  constexpr int CH = 16 * L;     // halves per chunk (one 32-byte load per lane of a subgroup)
  extern __shared__ __align__(128) unsigned char smem_raw[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool paired = (p.mode == kModePaired);
  const int nsegx = paired ? 2 : p.nseg;  // distinct gathered vectors
  const bool dense = (p.seg[0].idx == nullptr);

  // Row-group range of this CTA.
  const int g0 = (int)(((int64_t)blockIdx.x * p.row_groups) / gridDim.x);
  const int g1 = (int)(((int64_t)(blockIdx.x + 1) * p.row_groups) / gridDim.x);
  const int ng = g1 - g0;
  const int vgroups = paired ? 2 * ng : ng;

  // Shared memory carve-up (must match gemv_smem_bytes).
  const int max_vrows = (paired ? 2 : 1) * ((p.row_groups + gridDim.x - 1) / gridDim.x) * RG;
  const int w_al = (int)align_up_sz((size_t)p.w, 16);
  GemvSmem s;
  {
    size_t off = 0;
    s.xs = reinterpret_cast<__half*>(smem_raw + off);
    off += align_up_sz((size_t)p.K * 2, 16);
    s.sidx = reinterpret_cast<uint8_t*>(smem_raw + off);
    off += (size_t)w_al * nsegx;
    s.xc = reinterpret_cast<__half*>(smem_raw + off);
    off += align_up_sz((size_t)p.w_pad * 2 * nsegx, 16);
    s.acc = reinterpret_cast<float*>(smem_raw + off);
    off += align_up_sz((size_t)max_vrows * 4, 16);
    s.red = reinterpret_cast<float*>(smem_raw + off);
    off += 32 * 4;
    s.bar = reinterpret_cast<uint64_t*>(smem_raw + off);
  }

  // Work items of this warp: (virtual row-group, chunk) pairs t in [t0, t1).
  const int cpr = p.w_pad / CH;
  const int T = vgroups * cpr;
  const int t0 = (int)(((int64_t)warp * T) / kGemvWarps);
  const int t1 = (int)(((int64_t)(warp + 1) * T) / kGemvWarps);
  const int sub = lane / L, li = lane % L;

  // --- 1. Before the dependency wait (weights and masks never depend on an
  //        earlier kernel): start this warp's weight stream into registers,
  //        and start the bulk copies of the mask offsets.
  int l_vg = t0 / cpr, l_c = t0 - l_vg * cpr;  // load cursor
  const __half* l_ptr;
  bool l_valid;
  {
    const LaneRow r = lane_row(p, paired, g0, ng, l_vg, RG, sub);
    l_valid = r.valid;
    l_ptr = p.seg[r.segi].w + (size_t)r.lrow * p.w_pad + li * 16;
  }
  U32x8 buf[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (t0 + u < t1) {
      if (l_valid) {
        buf[u] = ld_stream_256(l_ptr + (size_t)l_c * CH);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) buf[u].v[e] = 0u;
      }
      if (++l_c == cpr) {
        l_c = 0;
        ++l_vg;
        const LaneRow r = lane_row(p, paired, g0, ng, l_vg, RG, sub);
        l_valid = r.valid;
        l_ptr = p.seg[r.segi].w + (size_t)r.lrow * p.w_pad + li * 16;
      }
    }
  }

  // L2 look-ahead beyond the register ring (lane 0 issues bulk prefetches of
  // whole chunk runs; every lane tracks the cursor so control stays uniform).
  auto pf_range = [&](int ta, int tb) {
    if (lane != 0) return;
    int vg = ta / cpr, c = ta - vg * cpr;
    while (ta < tb) {
      const int cend = min(cpr, c + (tb - ta));
#pragma unroll
      for (int sg = 0; sg < RG; ++sg) {
        const LaneRow r = lane_row(p, paired, g0, ng, vg, RG, sg);
        if (r.valid)
          bulk_prefetch_l2(p.seg[r.segi].w + (size_t)r.lrow * p.w_pad + (size_t)c * CH, (uint32_t)(cend - c) * CH * 2);
      }
      ta += cend - c;
      c = 0;
      ++vg;
    }
  };
  int pf_next = min(t1, t0 + U);
  if (p.pf_items > 0) {
    const int e = min(t1, pf_next + p.pf_items);
    pf_range(pf_next, e);
    pf_next = e;
  }

  const bool idx_bulk = !dense && ((p.w & 15) == 0);
  const bool x_bulk = (p.prologue == kProPlain) && ((reinterpret_cast<uintptr_t>(p.x) & 15u) == 0) &&
                      ((p.K & 7) == 0);
  if (tid == 0) {
    mbar_init(&s.bar[0], 1);
    mbar_init(&s.bar[1], 1);
    if (idx_bulk) {
      bool ok = true;
      for (int sx = 0; sx < nsegx; ++sx) ok = ok && ((reinterpret_cast<uintptr_t>(p.seg[sx].idx) & 15u) == 0);
      if (ok) {
        mbar_arrive_expect_tx(&s.bar[0], (uint32_t)(p.w * nsegx));
        for (int sx = 0; sx < nsegx; ++sx) bulk_copy_g2s(s.sidx + (size_t)sx * w_al, p.seg[sx].idx, (uint32_t)p.w, &s.bar[0]);
      } else {
        mbar_arrive_expect_tx(&s.bar[0], 0);
      }
    }
    // This CTA's share of the next launch's first weights, into L2.
    prefetch_shares_l2(p.next_pf, p.next_pf_bytes, p.next_pf_head, blockIdx.x, gridDim.x);
  }
  for (int v = tid; v < vgroups * RG; v += kGemvThreads) s.acc[v] = 0.f;
  __syncthreads();  // barrier init visible before anyone polls it
  bool idx_staged = false;
  if (idx_bulk) {
    bool ok = true;
    for (int sx = 0; sx < nsegx; ++sx) ok = ok && ((reinterpret_cast<uintptr_t>(p.seg[sx].idx) & 15u) == 0);
    idx_staged = ok;
  }

  // --- 2. Wait for the producer of x (no-op without programmatic launch).
  grid_dep_wait();

  // --- 3. Stage x in shared memory.
  const __half* xsrc = input_row(p);
  float rstd = 1.f;
  if (x_bulk) {
    if (tid == 0) {
      mbar_arrive_expect_tx(&s.bar[1], (uint32_t)p.K * 2);
      bulk_copy_g2s(s.xs, xsrc, (uint32_t)p.K * 2, &s.bar[1]);
    }
  } else {
    float ss = 0.f;
    const bool vec = ((p.K & 7) == 0) && ((reinterpret_cast<uintptr_t>(xsrc) & 15u) == 0) &&
                     (p.x2 == nullptr || (reinterpret_cast<uintptr_t>(p.x2) & 15u) == 0);
    if (vec) {
      // 16-byte pieces: one load of x (and x2) per thread for K <= 4096.
      for (int i8 = tid; i8 < p.K / 8; i8 += kGemvThreads) {
        const uint4 a = *reinterpret_cast<const uint4*>(xsrc + (size_t)i8 * 8);
        uint4 b = make_uint4(0u, 0u, 0u, 0u);
        const bool add = (p.prologue == kProResidNorm && p.x2 != nullptr);
        if (add) b = *reinterpret_cast<const uint4*>(p.x2 + (size_t)i8 * 8);
        const __half* ah = reinterpret_cast<const __half*>(&a);
        const __half* bh = reinterpret_cast<const __half*>(&b);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const __half hv = add ? f2h(h2f(ah[e]) + h2f(bh[e])) : ah[e];
          oh[e] = hv;
          const float vr = h2f(hv);
          ss = fmaf(vr, vr, ss);
        }
        *reinterpret_cast<uint4*>(s.xs + (size_t)i8 * 8) = o;
      }
    } else {
      for (int i = tid; i < p.K; i += kGemvThreads) {
        float v = h2f(xsrc[i]);
        if (p.prologue == kProResidNorm && p.x2 != nullptr) v = h2f(f2h(v + h2f(p.x2[i])));
        const __half hv = f2h(v);
        s.xs[i] = hv;
        const float vr = h2f(hv);
        ss = fmaf(vr, vr, ss);
      }
    }
    if (p.prologue == kProResidNorm) {
      const float tot = block_reduce_sum(ss, s.red);
      rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
    }
    __syncthreads();
    if (p.prologue == kProResidNorm && p.resid_out != nullptr && blockIdx.x == 0) {
      for (int i = tid; i < p.K; i += kGemvThreads) p.resid_out[i] = s.xs[i];
    }
  }
  bool ok = true;
  if (idx_staged) ok = mbar_wait_bounded(&s.bar[0], 0, 500ull * 1000 * 1000);
  if (x_bulk) ok = mbar_wait_bounded(&s.bar[1], 0, 500ull * 1000 * 1000) && ok;
  if (__syncthreads_or(!ok)) {
    // A bulk copy did not complete in time (error recorded).  Give the copies
    // one more bounded wait so nothing lands in shared memory after exit,
    // then skip the work.
    if (idx_staged) mbar_wait_bounded(&s.bar[0], 0, 500ull * 1000 * 1000);
    if (x_bulk) mbar_wait_bounded(&s.bar[1], 0, 500ull * 1000 * 1000);
    __syncthreads();
    return;
  }

  // --- 4. Gather xc for each distinct mask (permuted for conflict-free reads).
  for (int sx = 0; sx < nsegx; ++sx) {
    const uint8_t* idx = idx_staged ? (s.sidx + (size_t)sx * w_al) : p.seg[sx].idx;
    __half* xc = s.xc + (size_t)sx * p.w_pad;
    for (int j = tid; j < p.w_pad; j += kGemvThreads) {
      __half val = __ushort_as_half((unsigned short)0);
      if (j < p.w) {
        const int col = dense ? j : (j / p.n) * p.m + (int)idx[j];
        if (col < p.K) {
          val = s.xs[col];
          if (p.prologue == kProResidNorm) {
            const __half nrm = f2h(h2f(val) * rstd);
            val = f2h(h2f(nrm) * h2f(p.norm_w[col]));
          }
        }
      }
      xc[xc_perm<L>(j)] = val;
    }
  }
  __syncthreads();

  // Let the next kernel in the stream start its own pre-wait phase.
  grid_dep_launch_dependents();

  // --- 5. Stream weights through the register ring.  A warp accumulates
  //        while it stays on one row-group and flushes (L-lane reduction +
  //        shared atomic) when it leaves it or runs out of items.
  int c_vg = t0 / cpr, c_c = t0 - c_vg * cpr;  // consume cursor
  const __half* xcs;
  bool c_valid;
  {
    const LaneRow r = lane_row(p, paired, g0, ng, c_vg, RG, sub);
    c_valid = r.valid;
    xcs = s.xc + (size_t)r.segi * p.w_pad + li * 8;
  }
  float a0 = 0.f, a1 = 0.f;
  for (int base = t0; base < t1; base += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u;
      if (t < t1) {
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
        // Refill this ring slot U items ahead.
        if (t + U < t1) {
          if (l_valid) {
            buf[u] = ld_stream_256(l_ptr + (size_t)l_c * CH);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) buf[u].v[e] = 0u;
          }
          if (++l_c == cpr) {
            l_c = 0;
            ++l_vg;
            const LaneRow r = lane_row(p, paired, g0, ng, l_vg, RG, sub);
            l_valid = r.valid;
            l_ptr = p.seg[r.segi].w + (size_t)r.lrow * p.w_pad + li * 16;
          }
        }
        if (p.pf_items > 0 && pf_next < t1 && pf_next - t <= U + p.pf_items / 2) {
          const int e = min(t1, pf_next + max(1, p.pf_items / 2));
          pf_range(pf_next, e);
          pf_next = e;
        }
        // Advance the consume cursor; flush at the end of a row-group or range.
        const bool row_end = (++c_c == cpr);
        if (row_end || t + 1 == t1) {
          const float tot = group_reduce_sum<L>(a0 + a1);
          if (li == 0 && c_valid) atomicAdd(&s.acc[c_vg * RG + sub], tot);
          a0 = a1 = 0.f;
          if (row_end) {
            c_c = 0;
            ++c_vg;
            if (c_vg < vgroups) {
              const LaneRow r = lane_row(p, paired, g0, ng, c_vg, RG, sub);
              c_valid = r.valid;
              xcs = s.xc + (size_t)r.segi * p.w_pad + li * 8;
            }
          }
        }
      }
    }
  }
  __syncthreads();

  // --- 6. Epilogue over this CTA's rows.
  gemv_epilogue<kGemvThreads>(p, s.acc, g0, ng, RG, blockIdx.x, gridDim.x);
}

// ---------------------------------------------------------------------------
// Reference-layout kernel: mat_data[w, h], element (j, r) at j*h + r.
// A CTA owns RB = 16*LR consecutive rows (each lane accumulates 16 rows from
// one 32-byte load) and a slice of the compressed width; the CS CTAs of a
// thread-block cluster split the width and reduce through distributed shared
// memory into cluster rank 0, which writes fp16 output.  No atomics, no
// zero-fill, no fp32 scratch (reference: triton_spmv.py:285, :110-115).
// ---------------------------------------------------------------------------
struct GemvRefParams {
  const __half* vec;
  const __half* mat_data;
  const uint8_t* mat_index;
  __half* out;
  int32_t K, w, h, n, m;
  int32_t jchunk;  // compressed columns per cluster rank
  int32_t cs;      // cluster size (1 = no cluster)
};

__device__ __forceinline__ uint4 ld_stream_128(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// One weight element (row = lane's 16 rows, e) of a per-row layout: the
// gathered input is x[(j / N) * M + index byte e].
__device__ __forceinline__ void fma_rowwise16(float (&acc)[16], const U32x8& wv, const uint4& iv, const __half* xs,
                                              int gbase) {
  const uint8_t* ib = reinterpret_cast<const uint8_t*>(&iv);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&wv.v[e]));
    acc[2 * e] = fmaf(wf.x, h2f(xs[gbase + ib[2 * e]]), acc[2 * e]);
    acc[2 * e + 1] = fmaf(wf.y, h2f(xs[gbase + ib[2 * e + 1]]), acc[2 * e + 1]);
  }
}

// Reference layout [w, h]: lanes own 16 consecutive rows, warps and cluster
// ranks split the compressed width j.  ROW = false: shared mask
// (mat_index [w/N, N]), the gathered vector xc[j] is built once per CTA.
// ROW = true: per-row mask (mat_index [w, h], the reference's non-shared
// layout, src/spmv/nmsparse_linear.py:27-29): the full input vector is staged
// and every element gathers its own column.
template <int LR, bool ROW>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_ref_kernel(const __grid_constant__ GemvRefParams p) {
  constexpr int RB = 16 * LR;
  constexpr int JPW = kWarp / LR;           // j rows per warp instruction
  constexpr int JL = kGemvWarps * JPW;      // j lanes per CTA
  constexpr int U = 4;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __half* xc = reinterpret_cast<__half*>(smem_raw);  // [jchunk] (ROW: [K + 256], zero tail)
  const size_t xbytes = align_up_sz((size_t)(ROW ? p.K + 256 : p.jchunk) * 2, 16);
  float* red = reinterpret_cast<float*>(smem_raw + xbytes);  // [kGemvWarps][RB]
  float* part = red + kGemvWarps * RB;  // [RB]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rb = blockIdx.x;
  const int rank = blockIdx.y;
  const int j0 = rank * p.jchunk;
  const int j1 = min(p.w, j0 + p.jchunk);

  grid_dep_wait();
  if (ROW) {
    // An index byte is at most 255 past its group start: the zero tail keeps
    // every gather inside shared memory whatever the mask holds.
    for (int k = tid; k < p.K + 256; k += kGemvThreads) xc[k] = k < p.K ? p.vec[k] : __ushort_as_half((unsigned short)0);
  } else {
    for (int j = j0 + tid; j < j1; j += kGemvThreads) {
      const int col = (j / p.n) * p.m + (int)p.mat_index[j];
      xc[j - j0] = (col < p.K) ? p.vec[col] : __ushort_as_half((unsigned short)0);
    }
  }
  __syncthreads();
  grid_dep_launch_dependents();

  const int q = warp * JPW + lane / LR;  // j lane
  const int li = lane % LR;
  const int row0 = rb * RB + li * 16;
  const bool row_ok = row0 < p.h;  // h % 16 == 0 is enforced by the host
  float acc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) acc[k] = 0.f;

  const __half* base = p.mat_data + row0;
  const uint8_t* ibase = p.mat_index + row0;  // ROW: index bytes of the lane's rows
  int j = j0 + q;
  for (; j + (U - 1) * JL < j1; j += U * JL) {
    U32x8 r[U];
    uint4 ix[ROW ? U : 1];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (row_ok) {
        r[u] = ld_stream_256(base + (size_t)(j + u * JL) * p.h);
        if (ROW) ix[u] = ld_stream_128(ibase + (size_t)(j + u * JL) * p.h);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) r[u].v[e] = 0u;
        if (ROW) ix[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (ROW) {
        fma_rowwise16(acc, r[u], ix[u], xc, ((j + u * JL) / p.n) * p.m);
      } else {
        const uint16_t xh = __half_as_ushort(xc[j + u * JL - j0]);
#pragma unroll
        for (int e = 0; e < 8; ++e) fma2_f32_f16_bcast(acc[2 * e], acc[2 * e + 1], r[u].v[e], xh);
      }
    }
  }
  for (; j < j1; j += JL) {
    U32x8 r;
    uint4 ix = make_uint4(0u, 0u, 0u, 0u);
    if (row_ok) {
      r = ld_stream_256(base + (size_t)j * p.h);
      if (ROW) ix = ld_stream_128(ibase + (size_t)j * p.h);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) r.v[e] = 0u;
    }
    if (ROW) {
      fma_rowwise16(acc, r, ix, xc, (j / p.n) * p.m);
    } else {
      const uint16_t xh = __half_as_ushort(xc[j - j0]);
#pragma unroll
      for (int e = 0; e < 8; ++e) fma2_f32_f16_bcast(acc[2 * e], acc[2 * e + 1], r.v[e], xh);
    }
  }

  // Reduce across the JPW j-subgroups of the warp.
#pragma unroll
  for (int o = 16; o >= LR; o >>= 1) {
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  }
  if (lane < LR) {
#pragma unroll
    for (int k = 0; k < 16; ++k) red[warp * RB + li * 16 + k] = acc[k];
  }
  __syncthreads();
  for (int r = tid; r < RB; r += kGemvThreads) {
    float v = 0.f;
#pragma unroll 4
    for (int w2 = 0; w2 < kGemvWarps; ++w2) v += red[w2 * RB + r];
    part[r] = v;
  }
  if (p.cs > 1) {
    cluster_sync_all();
    if (rank == 0) {
      for (int r = tid; r < RB; r += kGemvThreads) {
        float v = part[r];
        for (int q2 = 1; q2 < p.cs; ++q2) v += ld_dsmem_f32(&part[r], (uint32_t)q2);
        const int row = rb * RB + r;
        if (row < p.h) p.out[row] = f2h(v);
      }
    }
    cluster_sync_all();  // keep every rank's shared memory alive until rank 0 has read it
  } else {
    __syncthreads();
    for (int r = tid; r < RB; r += kGemvThreads) {
      const int row = rb * RB + r;
      if (row < p.h) p.out[row] = f2h(part[r]);
    }
  }
}

// ---------------------------------------------------------------------------
// Layout conversion: reference [w, h]  <->  packed [h, w_pad] (zero padded).
// 32x32 tiles through shared memory.
// ---------------------------------------------------------------------------
__global__ void pack_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int w, int h,
                            int w_pad) {
  __shared__ __half tile[32][33];
  const int jb = blockIdx.x * 32, rb = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  grid_dep_wait();
  for (int k = ty; k < 32; k += 8) {
    const int j = jb + k, r = rb + tx;
    tile[k][tx] = (j < w && r < h) ? src[(size_t)j * h + r] : __ushort_as_half((unsigned short)0);
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int r = rb + k, j = jb + tx;
    if (r < h && j < w_pad) dst[(size_t)r * w_pad + j] = tile[tx][k];
  }
}

__global__ void unpack_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int w, int h,
                              int w_pad) {
  __shared__ __half tile[32][33];
  const int jb = blockIdx.x * 32, rb = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  grid_dep_wait();
  for (int k = ty; k < 32; k += 8) {
    const int r = rb + k, j = jb + tx;
    tile[k][tx] = (r < h && j < w) ? src[(size_t)r * w_pad + j] : __ushort_as_half((unsigned short)0);
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int j = jb + k, r = rb + tx;
    if (j < w && r < h) dst[(size_t)j * h + r] = tile[tx][k];
  }
}

}  // namespace nms
