// Standalone packed-layout GEMV with per-warp shared-memory weight rings.
//
// Same computation as gemv_packed_kernel (plain or residual + RMSNorm
// prologue; store, SwiGLU or argmax epilogue), laid out for back-to-back
// launches:
//
//   * one CTA per SM, at most half of an SM's registers and shared memory,
//     so the next launch's CTA fits beside it;
//   * every warp streams its weight items through its own ring of D 1 KB
//     slots with 16-byte cp.async copies (no registers held per byte in
//     flight: D = 8 keeps 96 KB per SM in flight at 12 warps; the deepest
//     ring of D = 8..4 that fits is used);
//   * the ring is filled and the mask offsets are staged BEFORE the
//     programmatic-dependency wait (weights never depend on an earlier
//     kernel), and the CTA lets its dependents launch at once.
//
// So while launch i streams its weights, launch i+1's CTAs are already
// resident and fill their rings; when launch i completes, launch i+1 only
// has to gather its input vector before it consumes weights that are
// already on chip.  The per-launch fixed cost (CTA start, first-load
// latency, input gather, tail) overlaps the neighbour's stream instead of
// leaving HBM idle.
//
// Determinism: a warp gets at least one row group of items, so a row is
// split over at most two warps and their two shared-memory partial sums add
// in either order to the same value (as in the persistent step).
#pragma once

#include "nms_common.cuh"
#include "nms_gemv.cuh"
#include "nms_step.cuh"

namespace nms {

constexpr int kRingThreads = 384;
constexpr int kRingWarps = kRingThreads / kWarp;
// Shared memory a CTA may take and still leave room for a second one on the
// SM (228 KB per SM, 1 KB reserved per CTA).
constexpr size_t kRingSmemCap = 112 * 1024;
// Weight bytes per SM above which a launch uses two CTAs per SM.
constexpr int64_t kRingTwoPerSmBytes = 256 * 1024;
// 16-byte input loads a thread keeps in flight while staging x.
constexpr int kRingStageLoads = 6;

__host__ __device__ inline size_t gemv_ring_smem_bytes(int D, int K, int w, int w_pad, int nsegx, int max_vrows,
                                                       bool norm) {
  size_t off = (size_t)kRingWarps * D * kRingItemBytes;
  off += align_up_sz((size_t)K * 2, 16) * (norm ? 2 : 1);
  off += align_up_sz((size_t)w, 16) * nsegx;
  off += align_up_sz((size_t)w_pad * 2 * nsegx, 16);
  off += align_up_sz((size_t)max_vrows * 4, 16);
  return off;
}

// NORM: the residual + RMSNorm prologue (a compile-time switch, so the plain
// launches keep the lean staging loop).
template <int L, int D, bool NORM>
__global__ void __launch_bounds__(kRingThreads, 2) gemv_ring_kernel(const __grid_constant__ GemvParams p) {
  constexpr int RG = kWarp / L, NT = kRingThreads, CB = 32 * L;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = lane / L, li = lane % L;
  const bool paired = (p.mode == kModePaired);
  const int nsegx = paired ? 2 : p.nseg;
  const bool dense = (p.seg[0].idx == nullptr);

  // Row groups of this CTA, items of this warp.
  const int g0 = (int)(((int64_t)blockIdx.x * p.row_groups) / gridDim.x);
  const int ng = (int)(((int64_t)(blockIdx.x + 1) * p.row_groups) / gridDim.x) - g0;
  const int vgroups = paired ? 2 * ng : ng;
  const int cpr = p.w_pad / (16 * L);
  const int T = vgroups * cpr;
  const int nw = max(1, min(kRingWarps, vgroups));
  int t0 = T, t1 = T;
  if (warp < nw) {
    t0 = (int)(((int64_t)warp * T) / nw);
    t1 = (int)(((int64_t)(warp + 1) * T) / nw);
  }

  const int w_al = (int)align_up_sz((size_t)p.w, 16);
  const int max_vrows = (paired ? 2 : 1) * ((p.row_groups + (int)gridDim.x - 1) / (int)gridDim.x) * RG;
  unsigned char* wring = smem_raw + (size_t)warp * D * kRingItemBytes;
  size_t off = (size_t)kRingWarps * D * kRingItemBytes;
  constexpr bool norm = NORM;
  __half* xs = reinterpret_cast<__half*>(smem_raw + off);
  off += align_up_sz((size_t)p.K * 2, 16);
  __half* nws = reinterpret_cast<__half*>(smem_raw + off);  // RMSNorm weight (norm prologue only)
  if (norm) off += align_up_sz((size_t)p.K * 2, 16);
  uint8_t* sidx = smem_raw + off;
  off += (size_t)w_al * nsegx;
  __half* xc = reinterpret_cast<__half*>(smem_raw + off);
  off += align_up_sz((size_t)p.w_pad * 2 * nsegx, 16);
  float* acc = reinterpret_cast<float*>(smem_raw + off);

  // --- 1. Fill the ring (items t0 .. t0 + D - 1; empty groups past t1).
  int pt = t0, pvg = t0 / cpr, pc = t0 - (t0 / cpr) * cpr, pslot = 0;
  const unsigned char* psrc = nullptr;
  bool pvalid = false;
  auto prow = [&]() {
    const LaneRow r = lane_row(p, paired, g0, ng, pvg, RG, sub);
    pvalid = r.valid;
    psrc = reinterpret_cast<const unsigned char*>(p.seg[r.segi].w + (size_t)r.lrow * p.w_pad) + li * 16 +
           (size_t)pc * CB;
  };
  auto produce = [&]() {
    if (pt < t1) {
      if (pvalid) {
        unsigned char* dst = wring + pslot * kRingItemBytes + lane * 16;
        cp_async_16(dst, psrc);
        cp_async_16(dst + 512, psrc + CB / 2);
      }
      ++pt;
      psrc += CB;
      if (++pc == cpr) {
        pc = 0;
        ++pvg;
        if (pt < t1) prow();
      }
      pslot = (pslot + 1 == D) ? 0 : pslot + 1;
    }
    cp_async_commit();
  };
  if (t0 < t1) prow();
#pragma unroll
  for (int k = 0; k < D; ++k) produce();

  // The next launch may start now: its CTAs fit beside this one and fill
  // their own rings while this CTA streams.
  grid_dep_launch_dependents();

  // --- 2. Mask offsets and RMSNorm weights (independent of the predecessor).
  if (norm) {
    if ((p.K & 7) == 0 && (reinterpret_cast<uintptr_t>(p.norm_w) & 15u) == 0) {
      for (int i = tid; i < p.K / 8; i += NT)
        reinterpret_cast<uint4*>(nws)[i] = __ldg(reinterpret_cast<const uint4*>(p.norm_w) + i);
    } else {
      for (int i = tid; i < p.K; i += NT) nws[i] = p.norm_w[i];
    }
  }
  if (!dense) {
    for (int sx = 0; sx < nsegx; ++sx) {
      const uint8_t* src = p.seg[sx].idx;
      uint8_t* dst = sidx + (size_t)sx * w_al;
      if ((p.w & 15) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        for (int i = tid; i < p.w / 16; i += NT)
          reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
      } else {
        for (int i = tid; i < p.w; i += NT) dst[i] = src[i];
      }
    }
  }
  for (int v = tid; v < max_vrows; v += NT) acc[v] = 0.f;
  __syncthreads();

  // --- 3. Wait for the producer of x, stage it in shared memory (16-byte
  //        L2 reads, every load of a thread issued before any is used), then
  //        gather the compressed vector(s) from there.
  grid_dep_wait();
  const __half* xsrc = input_row(p);
  const bool add = norm && p.x2 != nullptr;
  float ss = 0.f;
  if ((p.K & 7) == 0 && (reinterpret_cast<uintptr_t>(xsrc) & 15u) == 0 &&
      (!add || (reinterpret_cast<uintptr_t>(p.x2) & 15u) == 0)) {
    const int K8 = p.K >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(xsrc);
    const uint4* x2v = reinterpret_cast<const uint4*>(p.x2);
    for (int base = tid; base < K8; base += kRingStageLoads * NT) {
      uint4 a[kRingStageLoads], b[kRingStageLoads];
#pragma unroll
      for (int u = 0; u < kRingStageLoads; ++u) {
        const int i8 = base + u * NT;
        a[u] = b[u] = make_uint4(0u, 0u, 0u, 0u);
        if (i8 < K8) {
          a[u] = __ldcg(xv + i8);
          if (add) b[u] = __ldcg(x2v + i8);
        }
      }
#pragma unroll
      for (int u = 0; u < kRingStageLoads; ++u) {
        const int i8 = base + u * NT;
        if (i8 >= K8) break;
        if (norm) {
          // fp16(x + x2) as the reference's residual add rounds it; the
          // statistic over the rounded values.
          const __half* ah = reinterpret_cast<const __half*>(&a[u]);
          const __half* bh = reinterpret_cast<const __half*>(&b[u]);
          uint4 o;
          __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const __half hv = add ? f2h(h2f(ah[e]) + h2f(bh[e])) : ah[e];
            oh[e] = hv;
            ss = fmaf(h2f(hv), h2f(hv), ss);
          }
          a[u] = o;
        }
        reinterpret_cast<uint4*>(xs)[i8] = a[u];
      }
    }
  } else {
    for (int i = tid; i < p.K; i += NT) {
      __half hv = xsrc[i];
      if (add) hv = f2h(h2f(hv) + h2f(p.x2[i]));
      xs[i] = hv;
      ss = fmaf(h2f(hv), h2f(hv), ss);
    }
  }
  float rstd = 1.f;
  if (norm) {
    __shared__ float red[kRingWarps];
    const float tot = block_reduce_sum(ss, red);  // its barriers also publish xs
    rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
    if (p.resid_out != nullptr && blockIdx.x == 0)
      for (int i = tid; i < p.K; i += NT) p.resid_out[i] = xs[i];
  } else {
    __syncthreads();
  }
  const int n_shift = ((p.n & (p.n - 1)) == 0) ? __ffs(p.n) - 1 : -1;
  const int wq = p.w_pad >> 2;
  for (int sx = 0; sx < nsegx; ++sx) {
    const uint8_t* idx = sidx + (size_t)sx * w_al;
    __half* xcs = xc + (size_t)sx * p.w_pad;
    for (int q = tid; q < wq; q += NT) {
      const int j0 = q << 2;
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
            val = xs[col];
            if (norm) val = f2h(h2f(f2h(h2f(val) * rstd)) * h2f(nws[col]));
          }
        }
        v[e] = val;
      }
      *reinterpret_cast<uint2*>(xcs + j0) = *reinterpret_cast<const uint2*>(v);
    }
  }
  __syncthreads();

  // --- 4. Consume this warp's items; each consumed item commits the next copy.
  if (t0 < t1) {
    int vg = t0 / cpr, c = t0 - vg * cpr, cslot = 0;
    LaneRow r = lane_row(p, paired, g0, ng, vg, RG, sub);
    const unsigned char* xr = reinterpret_cast<const unsigned char*>(xc + (size_t)r.segi * p.w_pad) + li * 16;
    float a0 = 0.f, a1 = 0.f;
    for (int t = t0; t < t1; ++t) {
      cp_async_wait<D - 1>();
      const unsigned char* slot = wring + cslot * kRingItemBytes + lane * 16;
      const uint4 wa = *reinterpret_cast<const uint4*>(slot);
      const uint4 wb = *reinterpret_cast<const uint4*>(slot + 512);
      const uint4 xa = *reinterpret_cast<const uint4*>(xr + c * CB);
      const uint4 xb = *reinterpret_cast<const uint4*>(xr + c * CB + CB / 2);
      fma2_f32_f16(a0, a1, wa.x, xa.x);
      fma2_f32_f16(a0, a1, wa.y, xa.y);
      fma2_f32_f16(a0, a1, wa.z, xa.z);
      fma2_f32_f16(a0, a1, wa.w, xa.w);
      fma2_f32_f16(a0, a1, wb.x, xb.x);
      fma2_f32_f16(a0, a1, wb.y, xb.y);
      fma2_f32_f16(a0, a1, wb.z, xb.z);
      fma2_f32_f16(a0, a1, wb.w, xb.w);
      cslot = (cslot + 1 == D) ? 0 : cslot + 1;
      produce();
      if (++c == cpr || t + 1 == t1) {
        const float tot = group_reduce_sum<L>(a0 + a1);
        if (li == 0 && r.valid) atomicAdd(&acc[vg * RG + sub], tot);
        a0 = a1 = 0.f;
        if (c == cpr && t + 1 < t1) {
          c = 0;
          ++vg;
          r = lane_row(p, paired, g0, ng, vg, RG, sub);
          xr = reinterpret_cast<const unsigned char*>(xc + (size_t)r.segi * p.w_pad) + li * 16;
        }
      }
    }
  }
  cp_async_wait<0>();  // the trailing (empty) groups
  __syncthreads();

  // --- 5. Epilogue over this CTA's rows.
  gemv_epilogue<NT>(p, acc, g0, ng, RG, blockIdx.x, gridDim.x);
}

}  // namespace nms
