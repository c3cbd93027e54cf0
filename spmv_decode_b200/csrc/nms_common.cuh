// Device helpers shared by every nmsparse-b200 kernel (sm_100a only).
//
// Everything here is hand-written inline PTX or plain CUDA; nothing is taken
// from a library.  The kernels are compiled into one translation unit
// (nms_lib.cu), so file-scope __device__ state below is a single object.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nmsparse-b200 kernels target sm_100a only"
#endif

namespace nms {

constexpr int kWarp = 32;

// Device error word.  Bounded waits that give up set a nonzero code here and
// return instead of hanging; the host reads it with nms_device_error().
enum DeviceError : int {
  kDevOk = 0,
  kDevBulkCopyTimeout = 1,   // mbarrier wait on a bulk copy ran past its limit
  kDevBadPosition = 2,       // attention: token position outside the KV cache
  kDevBarrierTimeout = 3,    // persistent step: a grid barrier wait ran past its limit
  kDevRingTimeout = 4,       // persistent step: a weight-ring slot was never refilled
  kDevRingMismatch = 5,      // persistent step: a weight-ring chunk does not fit its stage
  kDevMmaTimeout = 6,        // prefill GEMM: a copy or tensor-core wait ran past its limit
};
__device__ int g_device_error;

__device__ __forceinline__ void set_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  A kernel launched with the
// programmatic-stream-serialization attribute may start while its
// predecessor is still running; grid_dep_wait() blocks until the predecessor
// grid has completed and its writes are visible.  Every kernel of this
// library calls grid_dep_wait() before it reads data produced by an earlier
// kernel and before its first global write, so the ordering guarantee is
// transitive along a chain of such launches.  Both are no-ops for a launch
// without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Streaming loads.  Weights are read exactly once per decode step, so they
// bypass L1 and are marked evict-first in L2 (keeps activations, KV cache and
// the next kernel's prefetched lines resident).  sm_100 supports 256-bit
// per-thread global loads; the L2 eviction-priority qualifier requires them.
// ---------------------------------------------------------------------------
struct U32x8 {
  uint32_t v[8];
};

__device__ __forceinline__ U32x8 ld_stream_256(const void* p) {
  U32x8 r;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]),
        "=r"(r.v[4]), "=r"(r.v[5]), "=r"(r.v[6]), "=r"(r.v[7])
      : "l"(p));
  return r;
}

// Bulk L2 prefetch through the TMA unit: one instruction covers `bytes`
// (multiple of 16, 16-byte aligned address).  Used before grid_dep_wait() to
// pull the first part of a kernel's weight stream into L2 while the previous
// kernel is still finishing.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
               : "memory");
}

// Cross-launch L2 prefetch: each of the two byte ranges (the next launch's
// weights) is split into `nb` equal shares, and CTA `b` prefetches the first
// `head` bytes of its share of each range -- the bytes the next launch's CTA
// `b` reads first when both grids partition the rows the same way.  Pieces
// are 16-byte aligned (ranges are whole packed rows) and at most 64 KB.
__device__ __forceinline__ void prefetch_shares_l2(const char* const (&ptr)[2], const uint32_t (&bytes)[2],
                                                   uint32_t head, unsigned b, unsigned nb) {
  if (head == 0) return;
  for (int r = 0; r < 2; ++r) {
    if (ptr[r] == nullptr || bytes[r] == 0) continue;
    const uint64_t len = bytes[r];
    const uint64_t lo = (len * b / nb) & ~15ull;
    const uint64_t hi = (b + 1 == nb) ? len : ((len * (b + 1) / nb) & ~15ull);
    const uint64_t e = hi < lo + head ? hi : lo + head;
    for (uint64_t q = lo; q + 16 <= e; q += 65536) {
      const uint64_t n = (e - q) < 65536 ? (e - q) : 65536;
      bulk_prefetch_l2(ptr[r] + q, (uint32_t)(n & ~15ull));
    }
  }
}

// ---------------------------------------------------------------------------
// Mixed-precision FMA: d = a*b + c with a, b fp16 and c, d fp32, one rounding
// (the fp16*fp16 product is exact in fp32, so this equals fmaf(float(a),
// float(b), c), the reference's fma.rn.f32 on converted operands).
// Two lanes of a packed half2 pair go to two accumulators for ILP.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fma2_f32_f16(float& acc0, float& acc1, uint32_t w2,
                                             uint32_t x2) {
  asm("{\n\t.reg .f16 wa, wb, xa, xb;\n\t"
      "mov.b32 {wa, wb}, %2;\n\t"
      "mov.b32 {xa, xb}, %3;\n\t"
      "fma.rn.f32.f16 %0, wa, xa, %0;\n\t"
      "fma.rn.f32.f16 %1, wb, xb, %1;\n\t}"
      : "+f"(acc0), "+f"(acc1)
      : "r"(w2), "r"(x2));
}

// Same x (broadcast) against both halves of a packed weight pair.
__device__ __forceinline__ void fma2_f32_f16_bcast(float& acc0, float& acc1, uint32_t w2,
                                                   uint16_t xh) {
  asm("{\n\t.reg .f16 wa, wb, xs;\n\t"
      "mov.b32 {wa, wb}, %2;\n\t"
      "mov.b16 xs, %3;\n\t"
      "fma.rn.f32.f16 %0, wa, xs, %0;\n\t"
      "fma.rn.f32.f16 %1, wb, xs, %1;\n\t}"
      : "+f"(acc0), "+f"(acc1)
      : "r"(w2), "h"(xh));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk global->shared copy (TMA, non-tensor, this CTA only).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst_smem, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase.  Gives up after `limit_ns` of global
// time, records kDevBulkCopyTimeout and returns false.  A bulk copy moves a
// few tens of KB, so the limit (hundreds of ms) is only reached if the copy
// engine has failed.
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;  // common case: no timer read
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) {
      set_device_error(kDevBulkCopyTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Thread-block cluster helpers (distributed shared memory reduction).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(const float* local_ptr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local_ptr)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Atomic add with acquire-release semantics at GPU scope (one round trip):
// publishes the writes this thread has observed (including the CTA's, after
// a block barrier) and returns the previous value with acquire ordering.
__device__ __forceinline__ unsigned atom_add_acq_rel_u32(unsigned* p, unsigned v) {
  unsigned prev;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(prev) : "l"(p), "r"(v) : "memory");
  return prev;
}

// ---------------------------------------------------------------------------
// Counter-based random numbers for temperature sampling: Philox4x32-10
// (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011), ten rounds of two 32x32->64 multiplies with the round keys bumped
// by the Weyl constants.  Stateless: the same (key, counter) gives the same
// four words on any CTA, GPU or host restatement.
// ---------------------------------------------------------------------------
__host__ __device__ inline void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = (uint32_t)p1;
    c[2] = n2;
    c[3] = (uint32_t)p0;
  }
}

// Gumbel(0, 1) noise for vocabulary row `row` at token position `pos`:
// -log(-log(u)), u uniform in (0, 1) from the top 24 bits of the first
// Philox word.  argmax(logit / T + noise) is a sample of softmax(logit / T)
// -- the reference's exponential race argmax(probs / q), q ~ Exp(1)
// (generate.py:46-48), written with log(q) = log(-log(u)).
__device__ __forceinline__ float gumbel_noise(uint64_t seed, int64_t pos, int64_t row) {
  uint32_t c[4] = {(uint32_t)row, (uint32_t)pos, (uint32_t)((uint64_t)pos >> 32), 0x5EED5A3Bu};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const float u = ((float)(c[0] >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

// ---------------------------------------------------------------------------
// Small reductions.
// ---------------------------------------------------------------------------
template <int L>
__device__ __forceinline__ float group_reduce_sum(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_reduce_sum(float v) { return group_reduce_sum<32>(v); }

// Block-wide sum; `red` must hold >= blockDim.x/32 floats.  All threads get
// the result.
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_reduce_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_reduce_sum(t);
  return t;
}

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

}  // namespace nms
