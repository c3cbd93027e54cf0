// Batch > 1 (prefill) shared-mask N:M sparse GEMM on the packed layout.
//
// The reference runs every multi-token input through a dense F.linear
// (src/spmv/nmsparse_linear.py:55-68); its op refuses rows != 1
// (src/spmv/nmsparse_op.py:84-87).  With one mask shared by all output rows
// the sparse product is a dense GEMM over the compressed width w = K*N/M:
//   out[t, r] = sum_j packed[r, j] * xc[t, j],
//   xc[t, j]  = x[t, (j / N) * M + mat_index[j / N, j % N]]
// (the same sum as the GEMV, src/spmv/triton_spmv.py:81-108, for every t).
//
// Two kernels:
//   gather_xc_kernel  builds xc [T, w_pad] fp16 (zeros past w), casting x
//                     (fp16, bf16 or fp32) to fp16 the way the reference op
//                     casts its input.
//   gemm_nm_kernel    one CTA per (128 rows of h, BN tokens, k-split) tile on
//                     the 5th-generation tensor cores: TMA (128-byte swizzle)
//                     streams packed rows and xc rows into a ring of shared
//                     memory stages, one thread issues tcgen05.mma (M=128,
//                     N=BN, K=16, fp16 x fp16 -> fp32) into a TMEM
//                     accumulator, and all four warps read it back with
//                     tcgen05.ld.  Both operands are K-major: row r of the
//                     packed matrix is A's row, token t of xc is B's row.
//
// Split-K (when the tiles alone leave SMs idle): the S k-splits of one tile
// run as one thread-block cluster.  After a cluster barrier (every main loop
// done, so the shared-memory rings are free), each CTA pushes its fp32
// partial, 16 columns at a time, into the shared memory of the CTA that owns
// those columns (16-byte remote stores over distributed shared memory);
// after a second barrier each owner sums its columns over the S partials in
// split order (so the result does not depend on timing) and writes them.
//
// Every mbarrier wait is bounded (kGemmWaitNs); a wait that runs out records
// kDevMmaTimeout in the device error word and the CTA finishes without
// issuing further copies or MMAs.
#pragma once

#include <cuda.h>  // CUtensorMap (type only; the encoder is fetched at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "nms_common.cuh"

namespace nms {

constexpr int kGemmBM = 128;          // rows of h per tile (UMMA M)
constexpr int kGemmBK = 64;           // compressed columns per swizzle atom: one 128-byte row
constexpr int kGemmMaxAtoms = 2;      // atoms per pipeline stage
constexpr int kGemmThreads = 128;     // 4 warps: TMA producer, MMA issuer, TMEM owner, all epilogue
constexpr int kGemmMaxStages = 8;
constexpr int kGemmMaxBN = 256;       // UMMA N limit and TMA box limit
constexpr int kGemmOutPitch = kGemmBM + 8;  // halves per staged output row (272 B, 16-B aligned)
constexpr uint64_t kGemmWaitNs = 200ull * 1000 * 1000;

struct GemmParams {
  __half* out;           // [T, h] fp16
  int32_t T, h;
  int32_t bn;            // tokens per tile (multiple of 16, <= 256)
  int32_t atoms;         // 64-column atoms per stage (1 or 2)
  int32_t kblocks;       // stages covering w_pad: ceil(w_pad / (64 * atoms))
  int32_t splits;        // k-splits per tile (<= kblocks, <= 8): the cluster size along z
  int32_t stages;        // shared-memory ring depth
  uint32_t idesc;        // tcgen05 instruction descriptor
  uint32_t tmem_cols;    // TMEM columns allocated (power of 2, >= 32, >= bn)
  int32_t vec_out;       // 16-byte output stores allowed (h % 8 == 0, out aligned)
};

// ---------------------------------------------------------------------------
// Gather: one thread per 8 consecutive compressed columns of one token.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

template <typename TX>
__global__ void __launch_bounds__(256) gather_xc_kernel(const TX* __restrict__ x, const uint8_t* __restrict__ idx,
                                                        __half* __restrict__ xc, int32_t T, int32_t K, int32_t w,
                                                        int32_t w_pad, int32_t n, int32_t m) {
  // The GEMM that follows is launched as a programmatic dependent: let it
  // start its prologue and weight loads now (it waits for this grid before
  // it reads xc).
  grid_dep_launch_dependents();
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int32_t chunks = w_pad >> 3;
  if (gid >= (int64_t)T * chunks) return;
  const int32_t t = (int32_t)(gid / chunks);
  const int32_t j0 = (int32_t)(gid - (int64_t)t * chunks) * 8;
  const TX* xr = x + (int64_t)t * K;
  int32_t g = j0 / n, i = j0 - g * n;  // group and slot of j0, then stepped
  __align__(16) __half v[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int32_t j = j0 + q;
    float f = 0.f;
    if (j < w) f = to_f32(xr[g * m + idx[j]]);
    v[q] = __float2half_rn(f);
    if (++i == n) {
      i = 0;
      ++g;
    }
  }
  *reinterpret_cast<uint4*>(xc + (int64_t)t * w_pad + j0) = *reinterpret_cast<const uint4*>(v);
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA primitives (cta_group::1, this CTA only).
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor: K-major operand tile whose rows are 128
// bytes (64 fp16) with the 128-byte swizzle TMA writes; groups of 8 rows are
// 1024 bytes apart (stride byte offset), the leading byte offset is unused
// for swizzled K-major layouts (1), descriptor version 1, swizzle mode 2.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, N = bn, M = 128.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int m, int bn) {
  return (1u << 4) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before it has
// completed (and so has finished reading its shared-memory operands).
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 16 consecutive fp32 accumulator columns of this thread's TMEM lane; the
// wait is in the same asm block so no use of the registers can be scheduled
// before the load has landed.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-window address of `local` (an address in this CTA's shared memory)
// in cluster rank `rank`'s shared memory.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

__device__ __forceinline__ void st_dsmem_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (global_timer_ns() - t0 > kGemmWaitNs) {
      set_device_error(kDevMmaTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// The GEMM.  grid = (m tiles, n tiles, splits) with clusters of (1, 1,
// splits), 128 threads, dynamic shared memory = 1 KB alignment slack +
// stages x atoms x (16 KB A + bn x 128 B B).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_nm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemmParams p) {
  extern __shared__ uint8_t gemm_smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kGemmMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kGemmMaxStages];
  __shared__ __align__(8) uint64_t accum_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int32_t s_abort, s_issued, s_consumed;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * p.bn, split = blockIdx.z;
  const int kb0 = (int)((int64_t)p.kblocks * split / p.splits);
  const int kb1 = (int)((int64_t)p.kblocks * (split + 1) / p.splits);
  const int nk = kb1 - kb0;

  const uint32_t raw = smem_u32(gemm_smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  // Stage s: atoms x A tile [128 rows][128 B], then atoms x B tile [bn][128 B].
  const uint32_t a_atom = kGemmBM * 128u, b_atom = (uint32_t)p.bn * 128u;
  const uint32_t a_bytes = a_atom * (uint32_t)p.atoms;
  const uint32_t stage_bytes = a_bytes + b_atom * (uint32_t)p.atoms;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&accum_bar, 1);
    s_abort = 0;
    s_issued = 0;
    s_consumed = 0;
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 2) tmem_alloc(&tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0 && lane == 0) {
    // TMA producer.  A stage past w_pad (odd atom count) reads the zero fill.
    // The first ring's weight tiles are requested before the gather grid has
    // finished (this grid is its programmatic dependent); xc tiles only after.
    int i = 0, s = 0;
    uint32_t ph = 0;
    const int npre = nk < p.stages ? nk : p.stages;
    for (; i < npre; ++i) {
      const uint32_t sa = base + (uint32_t)i * stage_bytes;
      const int32_t kx = (kb0 + i) * kGemmBK * p.atoms;
      mbar_arrive_expect_tx(&full_bar[i], stage_bytes);
      for (int a = 0; a < p.atoms; ++a)
        tma_load_2d(sa + (uint32_t)a * a_atom, &tm_a, kx + a * kGemmBK, m0, smem_u32(&full_bar[i]));
    }
    grid_dep_wait();
    for (int j = 0; j < npre; ++j) {
      const uint32_t sb = base + (uint32_t)j * stage_bytes + a_bytes;
      const int32_t kx = (kb0 + j) * kGemmBK * p.atoms;
      for (int a = 0; a < p.atoms; ++a)
        tma_load_2d(sb + (uint32_t)a * b_atom, &tm_b, kx + a * kGemmBK, n0, smem_u32(&full_bar[j]));
    }
    if (npre == p.stages) {
      s = 0;
      ph = 1u;
    } else {
      s = npre;
    }
    for (; i < nk; ++i) {
      if (!gemm_wait(&empty_bar[s], ph ^ 1u)) {
        atomicExch(&s_abort, 1);
        break;
      }
      const uint32_t sa = base + (uint32_t)s * stage_bytes;
      const uint32_t bar = smem_u32(&full_bar[s]);
      const int32_t kx = (kb0 + i) * kGemmBK * p.atoms;
      mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
      for (int a = 0; a < p.atoms; ++a) {
        tma_load_2d(sa + (uint32_t)a * a_atom, &tm_a, kx + a * kGemmBK, m0, bar);
        tma_load_2d(sa + a_bytes + (uint32_t)a * b_atom, &tm_b, kx + a * kGemmBK, n0, bar);
      }
      if (++s == p.stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    s_issued = i;
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: 4 MMAs (K = 16 each) per 64-column atom; advancing K by 16
    // fp16 inside the 128-byte swizzle row is +32 bytes on the start address.
    int i = 0, s = 0;
    uint32_t ph = 0;
    for (; i < nk; ++i) {
      if (!gemm_wait(&full_bar[s], ph)) {
        atomicExch(&s_abort, 1);
        break;
      }
      tc_fence_after();
      const uint32_t sa = base + (uint32_t)s * stage_bytes;
      for (int a = 0; a < p.atoms; ++a) {
        const uint64_t da = umma_desc_k_sw128(sa + (uint32_t)a * a_atom);
        const uint64_t db = umma_desc_k_sw128(sa + a_bytes + (uint32_t)a * b_atom);
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk)
          umma_f16(tmem, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), p.idesc, (i | a | kk) != 0 ? 1u : 0u);
      }
      umma_commit(smem_u32(&empty_bar[s]));
      if (++s == p.stages) {
        s = 0;
        ph ^= 1u;
      }
    }
    s_consumed = i;
    umma_commit(smem_u32(&accum_bar));
  }
  __syncwarp();

  // ---- epilogue: TMEM lane (32 * warp + lane) holds tile row m0 + that ----
  const bool acc_ok = gemm_wait(&accum_bar, 0);
  tc_fence_after();
  __syncthreads();  // s_abort, s_issued and s_consumed are final
  if (threadIdx.x == 0 && s_abort) {
    // A wait of the main loop gave up (kDevMmaTimeout recorded): let the
    // tile copies still in flight land before the ring's shared memory is
    // reused below (split-K receive buffer, output staging).  Each wait is
    // bounded.  The cluster's output tile is then undefined -- it may be
    // unwritten or hold partial sums -- and the caller must treat the
    // launch's result as void.
    for (int i = s_consumed; i < s_issued; ++i) {
      if (!gemm_wait(&full_bar[i % p.stages], (uint32_t)(i / p.stages) & 1u)) break;
    }
  }
  __syncthreads();
  const int row = warp * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const int nchunks = p.bn >> 4;
  // Token range [t_begin, t_begin + t_count) of the tile this CTA writes,
  // staged as fp16 rows out_s[t][128 + 8 pad] before coalesced stores.
  __half* out_s = reinterpret_cast<__half*>(gemm_smem_raw + (base - raw));
  int t_begin = 0, t_count = p.bn;
  if (p.splits > 1) {
    // 16-column chunks of the tile are owned by cluster ranks in blocks of
    // cpr.  Every rank pushes each chunk of its partial into the owner's
    // receive buffer recv[split][128 rows][cpr * 16 columns + 4 pad] (four
    // 16-byte remote stores per thread and chunk); the owner then sums its
    // columns over the splits in split order.
    const int S = p.splits, r = (int)cluster_ctarank();
    const int cpr = (nchunks + S - 1) / S;
    const uint32_t pitch = (uint32_t)cpr * 16u + 4u;  // floats per receive row
    cluster_sync_all();  // every rank is past its main loop: the rings are free
    for (int c = 0; c < nchunks; ++c) {
      float v[16];
      tmem_ld16(trow + (uint32_t)(c * 16), v);
      const int q = c / cpr, lc = c - q * cpr;
      const uint32_t dst =
          dsmem_addr(base, (uint32_t)q) + (((uint32_t)r * kGemmBM + (uint32_t)row) * pitch + (uint32_t)lc * 16u) * 4u;
#pragma unroll
      for (int e = 0; e < 4; ++e) st_dsmem_v4(dst + 16u * e, v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    }
    cluster_sync_all();  // all pushes have landed
    const int c_first = r * cpr;
    const int c_end = min(nchunks, c_first + cpr);
    t_begin = c_first * 16;
    t_count = c_end > c_first ? (c_end - c_first) * 16 : 0;
    const float* recv = reinterpret_cast<const float*>(gemm_smem_raw + (base - raw));
    out_s = reinterpret_cast<__half*>(gemm_smem_raw + (base - raw) + (size_t)S * kGemmBM * pitch * 4);
    for (int lc = 0; lc * 16 < t_count; ++lc) {
      float acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0.f;
      for (int sp = 0; sp < S; ++sp) {
        const float4* src = reinterpret_cast<const float4*>(recv + ((size_t)sp * kGemmBM + row) * pitch + lc * 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 f = src[e];
          acc[4 * e] += f.x;
          acc[4 * e + 1] += f.y;
          acc[4 * e + 2] += f.z;
          acc[4 * e + 3] += f.w;
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) out_s[(lc * 16 + j) * kGemmOutPitch + row] = __float2half_rn(acc[j]);
    }
  } else {
    for (int c = 0; c < nchunks; ++c) {
      float v[16];
      tmem_ld16(trow + (uint32_t)(c * 16), v);
#pragma unroll
      for (int j = 0; j < 16; ++j) out_s[(c * 16 + j) * kGemmOutPitch + row] = __float2half_rn(v[j]);
    }
  }
  __syncthreads();
  if (acc_ok) {
    const int rows_valid = min(t_count, p.T - n0 - t_begin);
    const int cols_valid = min(kGemmBM, p.h - m0);
    for (int q = threadIdx.x; q < t_count * (kGemmBM / 8); q += kGemmThreads) {
      const int t = q >> 4, c8 = (q & 15) * 8;
      if (t >= rows_valid || c8 >= cols_valid) continue;
      __half* dst = p.out + (int64_t)(n0 + t_begin + t) * p.h + m0 + c8;
      const __half* src = out_s + t * kGemmOutPitch + c8;
      if (p.vec_out && c8 + 8 <= cols_valid) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      } else {
        const int e_end = min(8, cols_valid - c8);
        for (int e = 0; e < e_end; ++e) dst[e] = src[e];
      }
    }
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  // If the accumulator's commit never arrived, tensor-core work may still
  // write TMEM: give it one more bounded wait before the columns are freed.
  if (!acc_ok && warp == 2 && lane == 0) gemm_wait(&accum_bar, 0);
  __syncwarp();
  if (warp == 2) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace nms
