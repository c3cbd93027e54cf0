// libnmsparse_b200: C-ABI entry points for the B200 N:M sparse GEMV decode path.
//
// One translation unit: every kernel header is included here, so file-scope
// __device__ state (the device error word) exists once per loaded library.
// The ABI uses plain pointers, 64-bit sizes and an opaque stream handle
// (cudaStream_t passed as void*; nullptr = legacy default stream).  Every
// entry point validates its arguments, never aborts, and returns an
// nms_status code; nms_last_error() gives the message of the calling
// thread's last failure.
//
// Each launch is first turned into a frozen LaunchRec (kernel choice,
// parameters, grid, shared memory, launch attributes).  The direct entry
// points launch the record immediately; the plan API stores records and
// replays them (nms_plan_launch), which is the decode-step executor.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <type_traits>
#include <string>
#include <utility>
#include <vector>

#include "../../include/nmsparse_b200.h"

#include "nms_common.cuh"
#include "nms_decode.cuh"
#include "nms_gemm.cuh"
#include "nms_gemv.cuh"
#include "nms_step.cuh"
#include "nms_flow.cuh"
#include "nms_gemv_ring.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int fail_cuda(cudaError_t e, const char* what) {
  return fail(NMS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

constexpr int kMaxDevices = 64;
constexpr int kGemvCtasPerSm = 2;  // packed GEMV: two 512-thread CTAs per SM

struct DeviceInfo {
  bool ready = false;
  int num_sms = 0;
  size_t max_smem_optin = 0;
  size_t step_smem_max = 0;
  size_t gemm_smem_max = 0;  // dynamic shared memory gemm_nm_kernel may use
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// The ring GEMV instantiations of one ring depth (every lanes-per-row
// variant, both prologues).
#define NMS_RING_KERNELS_N(D, N)                                                                    \
  (const void*)nms::gemv_ring_kernel<32, D, N>, (const void*)nms::gemv_ring_kernel<16, D, N>,     \
      (const void*)nms::gemv_ring_kernel<8, D, N>, (const void*)nms::gemv_ring_kernel<4, D, N>
#define NMS_RING_KERNELS(D) NMS_RING_KERNELS_N(D, false), NMS_RING_KERNELS_N(D, true)

// Per-device one-time setup: SM count, opt-in shared memory, and the
// function attributes of every kernel instantiation.
int device_info(const DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NMS_ERR_VALUE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0, sms = 0, smem = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (major != 10 || minor != 0)
      return fail(NMS_ERR_NOT_IMPLEMENTED,
                  "libnmsparse_b200 is built for sm_100a (B200); device %d is sm_%d%d", dev, major, minor);
    d.num_sms = sms;
    d.max_smem_optin = (size_t)smem;
    const void* dyn_smem_kernels[] = {
        (const void*)nms::gemv_packed_kernel<32>, (const void*)nms::gemv_packed_kernel<16>,
        (const void*)nms::gemv_packed_kernel<8>,  (const void*)nms::gemv_packed_kernel<4>,
        (const void*)nms::gemv_ref_kernel<8, false>, (const void*)nms::gemv_ref_kernel<8, true>,
        NMS_RING_KERNELS(8), NMS_RING_KERNELS(6), NMS_RING_KERNELS(5), NMS_RING_KERNELS(4),
    };
    size_t static_max = 0;
    for (const void* k : dyn_smem_kernels) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, k);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncGetAttributes");
      if (fa.sharedSizeBytes > static_max) static_max = fa.sharedSizeBytes;
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
    }
    // The ring GEMV keeps its CTA at most half an SM so that the next
    // launch's CTA fits beside it: ask for the largest shared-memory carveout
    // (the default sizes the carveout for one CTA's need).
    for (const void* k : {NMS_RING_KERNELS(8), NMS_RING_KERNELS(6), NMS_RING_KERNELS(5), NMS_RING_KERNELS(4)}) {
      e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(PreferredSharedMemoryCarveout)");
    }
    // Dynamic shared memory available to every kernel that takes it.
    d.max_smem_optin = (size_t)smem - static_max;
    d.step_smem_max = (size_t)smem;
    for (const void* k : {(const void*)nms::decode_step_kernel<nms::kStepDepthHi>,
                          (const void*)nms::decode_step_kernel<nms::kStepDepthLo>,
                          (const void*)nms::decode_flow_kernel<nms::kStepDepthHi>,
                          (const void*)nms::decode_flow_kernel<nms::kStepDepthLo>}) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, k);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncGetAttributes(decode_step_kernel)");
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(decode_step_kernel)");
      d.step_smem_max = std::min(d.step_smem_max, (size_t)smem - fa.sharedSizeBytes);
    }
    {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, (const void*)nms::gemm_nm_kernel);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncGetAttributes(gemm_nm_kernel)");
      d.gemm_smem_max = (size_t)smem - fa.sharedSizeBytes;
      e = cudaFuncSetAttribute((const void*)nms::gemm_nm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)d.gemm_smem_max);
      if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(gemm_nm_kernel)");
    }
    e = cudaFuncSetAttribute((const void*)nms::attention_decode_kernel,
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(NonPortableClusterSizeAllowed)");
    d.ready = true;
  }
  *out = &d;
  return NMS_OK;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex2(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                       dim3 cluster, bool cooperative, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[3];
  int na = 0;
  if (cooperative) {
    attrs[na].id = cudaLaunchAttributeCooperative;
    attrs[na].val.cooperative = 1;
    ++na;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = cluster.x;
    attrs[na].val.clusterDim.y = cluster.y;
    attrs[na].val.clusterDim.z = cluster.z;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      dim3 cluster, Args&&... args) {
  return launch_ex2(kernel, grid, block, smem, st, pdl, cluster, false, std::forward<Args>(args)...);
}

struct EmbedParams {
  const __half* table;
  const int64_t* token;
  __half* x;
  int K;
  int64_t vocab;
};

// A frozen, validated launch.
struct LaunchRec {
  enum Kind { kGemvPacked, kGemvRef, kAttention, kEmbedding, kPack, kUnpack } kind;
  int lanes = 0;  // gemv_packed_kernel template argument
  int ring_depth = 0;  // > 0: gemv_ring_kernel with this ring depth (lanes as above)
  bool rowwise = false;  // kGemvRef: per-row mask (mat_index [w, h])
  int amax_capacity = 0;  // argmax epilogue: partials the caller's scratch holds
  nms::GemvParams gp;
  nms::GemvRefParams rp;
  nms::AttnParams ap;
  EmbedParams ep;
  struct {
    const __half* src;
    __half* dst;
    int w, h, w_pad;
  } pk;
  dim3 grid, block, cluster{1, 1, 1};
  size_t smem = 0;
  bool pdl = false;
};

template <int D, bool NORM>
cudaError_t launch_gemv_ring_d(const LaunchRec& r, cudaStream_t st) {
  switch (r.lanes) {
    case 32: return launch_ex(nms::gemv_ring_kernel<32, D, NORM>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp);
    case 16: return launch_ex(nms::gemv_ring_kernel<16, D, NORM>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp);
    case 8: return launch_ex(nms::gemv_ring_kernel<8, D, NORM>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp);
    default: return launch_ex(nms::gemv_ring_kernel<4, D, NORM>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp);
  }
}

template <bool NORM>
cudaError_t launch_gemv_ring_n(const LaunchRec& r, cudaStream_t st) {
  switch (r.ring_depth) {
    case 8: return launch_gemv_ring_d<8, NORM>(r, st);
    case 6: return launch_gemv_ring_d<6, NORM>(r, st);
    case 5: return launch_gemv_ring_d<5, NORM>(r, st);
    default: return launch_gemv_ring_d<4, NORM>(r, st);
  }
}

cudaError_t launch_gemv_ring(const LaunchRec& r, cudaStream_t st) {
  return r.gp.prologue == nms::kProResidNorm ? launch_gemv_ring_n<true>(r, st) : launch_gemv_ring_n<false>(r, st);
}

int launch_rec(const LaunchRec& r, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  switch (r.kind) {
    case LaunchRec::kGemvPacked:
      if (r.ring_depth > 0) {
        e = launch_gemv_ring(r, st);
        break;
      }
      switch (r.lanes) {
        case 32: e = launch_ex(nms::gemv_packed_kernel<32>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp); break;
        case 16: e = launch_ex(nms::gemv_packed_kernel<16>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp); break;
        case 8: e = launch_ex(nms::gemv_packed_kernel<8>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp); break;
        default: e = launch_ex(nms::gemv_packed_kernel<4>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.gp); break;
      }
      break;
    case LaunchRec::kGemvRef:
      e = r.rowwise ? launch_ex(nms::gemv_ref_kernel<8, true>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.rp)
                    : launch_ex(nms::gemv_ref_kernel<8, false>, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.rp);
      break;
    case LaunchRec::kAttention:
      e = launch_ex(nms::attention_decode_kernel, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.ap);
      break;
    case LaunchRec::kEmbedding:
      e = launch_ex(nms::embedding_kernel, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.ep.table, r.ep.token,
                    r.ep.x, r.ep.K, r.ep.vocab);
      break;
    case LaunchRec::kPack:
      e = launch_ex(nms::pack_kernel, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.pk.src, r.pk.dst, r.pk.w,
                    r.pk.h, r.pk.w_pad);
      break;
    case LaunchRec::kUnpack:
      e = launch_ex(nms::unpack_kernel, r.grid, r.block, r.smem, st, r.pdl, r.cluster, r.pk.src, r.pk.dst, r.pk.w,
                    r.pk.h, r.pk.w_pad);
      break;
  }
  if (e != cudaSuccess) return fail_cuda(e, "kernel launch");
  return NMS_OK;
}

int pick_lanes_per_row(int64_t w_pad) {
  for (int L = 32; L >= 4; L >>= 1)
    if (w_pad % (16 * L) == 0) return L;
  return 0;
}

// Shared validation of the N:M shape parameters (reference checks:
// triton_spmv.py:255-283, src/spmv/nmsparse_linear.py:39).
int check_nm(int64_t K, int64_t w, int32_t n, int32_t m) {
  if (n < 1 || m < 1) return fail(NMS_ERR_VALUE, "block_width=%d and vec_width=%d must be positive", n, m);
  if (n > m) return fail(NMS_ERR_VALUE, "block_width=%d must not exceed vec_width=%d", n, m);
  if (m > 256) return fail(NMS_ERR_VALUE, "vec_width=%d exceeds the uint8 in-group offset range", m);
  if (w <= 0 || K <= 0) return fail(NMS_ERR_VALUE, "w=%lld and K=%lld must be positive", (long long)w, (long long)K);
  if (w % n != 0) return fail(NMS_ERR_VALUE, "w=%lld must be divisible by N=%d", (long long)w, n);
  if ((w / n) * (int64_t)m != K)
    return fail(NMS_ERR_VALUE, "vector length K=%lld != (w/N)*M = %lld", (long long)K, (long long)((w / n) * m));
  if (K > (1 << 24)) return fail(NMS_ERR_VALUE, "K=%lld too large", (long long)K);
  return NMS_OK;
}

// Validate and copy a cross-launch prefetch description.
int fill_next_prefetch(const void* const (&src)[2], const int64_t (&bytes)[2], int64_t head, const char* (&dst)[2],
                       uint32_t (&dbytes)[2], uint32_t& dhead) {
  for (int r = 0; r < 2; ++r) {
    dst[r] = static_cast<const char*>(src[r]);
    if (bytes[r] < 0 || bytes[r] > 0xFFFFFFF0ll) return fail(NMS_ERR_VALUE, "next_prefetch_bytes[%d] out of range", r);
    if (src[r] == nullptr && bytes[r] != 0) return fail(NMS_ERR_VALUE, "next_prefetch[%d] is null", r);
    if (src[r] != nullptr && (!aligned(src[r], 16) || (bytes[r] & 15) != 0))
      return fail(NMS_ERR_VALUE, "next_prefetch[%d] must be 16-byte aligned with a multiple-of-16 size", r);
    dbytes[r] = (uint32_t)bytes[r];
  }
  if (head < 0 || head > (1 << 30)) return fail(NMS_ERR_VALUE, "next_prefetch_head out of range");
  dhead = (uint32_t)head;
  return NMS_OK;
}

// Build the record of a packed-layout GEMV launch (all fused variants).
int prepare_gemv(const nms_gemv_fused_args* a, LaunchRec* rec) {
  if (a == nullptr) return fail(NMS_ERR_VALUE, "args is null");
  if (a->nseg < 1 || a->nseg > NMS_MAX_SEGMENTS) return fail(NMS_ERR_VALUE, "nseg=%d out of range", a->nseg);
  if (!a->x || !a->out) return fail(NMS_ERR_VALUE, "null x or out pointer");
  const bool dense = (a->flags & NMS_FLAG_DENSE) != 0;
  int rc;
  if (dense) {
    if (a->w != a->K) return fail(NMS_ERR_VALUE, "dense launch needs w == K (w=%lld, K=%lld)", (long long)a->w, (long long)a->K);
    if (a->K <= 0 || a->K > (1 << 24)) return fail(NMS_ERR_VALUE, "bad K=%lld", (long long)a->K);
  } else {
    rc = check_nm(a->K, a->w, a->block_width, a->vec_width);
    if (rc) return rc;
  }
  for (int i = 0; i < a->nseg; ++i) {
    const nms_segment& s = a->seg[i];
    if (!dense && s.mat_index == nullptr) return fail(NMS_ERR_VALUE, "segment %d: null mat_index", i);
    if (dense && s.mat_index != nullptr) return fail(NMS_ERR_VALUE, "dense launch must not pass mat_index");
    if (s.packed == nullptr) return fail(NMS_ERR_VALUE, "segment %d: null weight pointer", i);
    if (!aligned(s.packed, 32)) return fail(NMS_ERR_VALUE, "segment %d: packed weights must be 32-byte aligned", i);
    if (s.rows <= 0) return fail(NMS_ERR_VALUE, "segment %d: rows must be positive", i);
  }
  int mode = nms::kModeConcat, epi = nms::kEpiStore, pro = nms::kProPlain;
  if (a->epilogue == NMS_EPI_SWIGLU) {
    mode = nms::kModePaired;
    epi = nms::kEpiSwiGLU;
  } else if (a->epilogue == NMS_EPI_ARGMAX) {
    epi = nms::kEpiArgmax;
    if (!a->amax_val || !a->amax_idx || !a->amax_counter || !a->token_out)
      return fail(NMS_ERR_VALUE, "argmax epilogue needs amax_val, amax_idx, amax_counter and token_out");
  } else if (a->epilogue != NMS_EPI_STORE) {
    return fail(NMS_ERR_VALUE, "unknown epilogue %d", a->epilogue);
  }
  if (a->prologue == NMS_PRO_RESID_RMSNORM) {
    pro = nms::kProResidNorm;
    if (!a->norm_weight) return fail(NMS_ERR_VALUE, "rmsnorm prologue needs norm_weight");
  } else if (a->prologue != NMS_PRO_PLAIN) {
    return fail(NMS_ERR_VALUE, "unknown prologue %d", a->prologue);
  }
  if (a->prefetch_bytes < 0) return fail(NMS_ERR_VALUE, "prefetch_bytes must be >= 0");

  const DeviceInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  const int64_t K = a->K, w = a->w, w_pad = a->w_pad;
  const int L = pick_lanes_per_row(w_pad);
  if (L == 0) return fail(NMS_ERR_VALUE, "packed row stride w_pad=%lld must be a multiple of 64", (long long)w_pad);
  if (w_pad < w) return fail(NMS_ERR_VALUE, "w_pad=%lld < w=%lld", (long long)w_pad, (long long)w);
  const int RG = 32 / L;

  nms::GemvParams& p = rec->gp;
  memset(&p, 0, sizeof(p));
  int64_t rows_total = 0;
  const bool paired = (mode == nms::kModePaired);
  for (int i = 0; i < a->nseg; ++i) {
    const nms_segment& s = a->seg[i];
    p.seg[i].w = static_cast<const __half*>(s.packed);
    p.seg[i].idx = static_cast<const uint8_t*>(s.mat_index);
    p.seg[i].rows = (int32_t)s.rows;
    p.seg[i].row_start = paired ? 0 : (int32_t)rows_total;
    if (!paired) rows_total += s.rows;
  }
  if (paired) {
    if (a->nseg != 2 || a->seg[0].rows != a->seg[1].rows)
      return fail(NMS_ERR_VALUE, "SwiGLU epilogue needs two segments (gate, up) with equal rows");
    rows_total = a->seg[0].rows;
  }
  if (rows_total > (1 << 30)) return fail(NMS_ERR_VALUE, "too many rows");
  p.nseg = a->nseg;
  p.mode = mode;
  p.prologue = pro;
  p.epilogue = epi;
  p.K = (int32_t)K;
  p.n = dense ? 1 : a->block_width;
  p.m = dense ? 1 : a->vec_width;
  p.w = (int32_t)w;
  p.w_pad = (int32_t)w_pad;
  p.rows_total = (int32_t)rows_total;
  p.row_groups = (int32_t)((rows_total + RG - 1) / RG);
  p.pf_items = a->prefetch_bytes / 1024;  // one work item streams 1 KB (32 lanes x 32 bytes)
  rc = fill_next_prefetch(a->next_prefetch, a->next_prefetch_bytes, a->next_prefetch_head, p.next_pf,
                          p.next_pf_bytes, p.next_pf_head);
  if (rc) return rc;
  p.x = static_cast<const __half*>(a->x);
  p.x2 = static_cast<const __half*>(a->x2);
  p.norm_w = static_cast<const __half*>(a->norm_weight);
  p.eps = a->eps;
  p.resid_out = static_cast<__half*>(a->resid_out);
  p.out = static_cast<__half*>(a->out);
  p.amax_val = a->amax_val;
  p.amax_idx = a->amax_idx;
  p.amax_counter = a->amax_counter;
  p.token_out = a->token_out;
  p.x_token = a->x_token;
  p.x_rows = a->x_rows;
  if (a->x_token != nullptr && a->x_rows <= 0) return fail(NMS_ERR_VALUE, "x_token needs x_rows > 0");
  p.next_token = a->next_token;
  p.token_history = a->token_history;
  p.pos = a->pos;
  p.history_len = a->history_len;
  if (epi != nms::kEpiArgmax && (a->next_token || a->token_history || a->pos))
    return fail(NMS_ERR_VALUE, "generation hooks need the argmax epilogue");
  if (!(a->temperature >= 0.f) || a->temperature > 1e30f)
    return fail(NMS_ERR_VALUE, "temperature must be finite and >= 0 (got %g)", (double)a->temperature);
  if (a->temperature > 0.f && epi != nms::kEpiArgmax)
    return fail(NMS_ERR_VALUE, "temperature sampling needs the argmax epilogue");
  p.temperature = a->temperature;
  p.sample_seed = a->sample_seed;
  p.sample_pos = a->sample_pos;
  p.sample_row_offset = a->sample_row_offset;

  int grid = a->grid > 0 ? a->grid : dev->num_sms * kGemvCtasPerSm;
  if (grid > p.row_groups) grid = p.row_groups;
  if (grid < 1) grid = 1;
  if (epi == nms::kEpiArgmax && grid > a->amax_capacity)
    return fail(NMS_ERR_VALUE, "argmax scratch holds %d partials, the launch needs %d", a->amax_capacity, grid);
  const int nsegx = paired ? 2 : a->nseg;
  const int max_vrows = (paired ? 2 : 1) * ((p.row_groups + grid - 1) / grid) * RG;
  const size_t smem = nms::gemv_smem_bytes((int)K, (int)w, (int)w_pad, nsegx, max_vrows);
  if (smem > dev->max_smem_optin)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "K=%lld, w_pad=%lld, %d masks need %zu bytes of shared memory (limit %zu)",
                (long long)K, (long long)w_pad, nsegx, smem, dev->max_smem_optin);
  rec->kind = LaunchRec::kGemvPacked;
  rec->lanes = L;
  rec->ring_depth = 0;
  if ((a->flags & NMS_FLAG_REGISTER_RING) == 0 && p.pf_items == 0) {
    // One CTA per SM, so that the next launch's CTA fits beside it; two when
    // the stream is long (over 256 KB of weights per SM), where more bytes in
    // flight pay more than the overlap with the neighbouring launches.
    int64_t wbytes = 0;
    for (int i = 0; i < a->nseg; ++i) wbytes += a->seg[i].rows * w_pad * 2;
    int rgrid = a->grid > 0 ? a->grid
                            : dev->num_sms * (wbytes > (int64_t)dev->num_sms * nms::kRingTwoPerSmBytes ? 2 : 1);
    if (rgrid > p.row_groups) rgrid = p.row_groups;
    if (rgrid < 1) rgrid = 1;
    const int rvrows = (paired ? 2 : 1) * ((p.row_groups + rgrid - 1) / rgrid) * RG;
    for (int D : {8, 6, 5, 4}) {
      const size_t rs = nms::gemv_ring_smem_bytes(D, (int)K, (int)w, (int)w_pad, nsegx, rvrows, pro == nms::kProResidNorm);
      if (rs <= nms::kRingSmemCap && rs <= dev->max_smem_optin &&
          !(epi == nms::kEpiArgmax && rgrid > a->amax_capacity)) {
        rec->ring_depth = D;
        rec->grid = dim3(rgrid);
        rec->block = dim3(nms::kRingThreads);
        rec->smem = rs;
        break;
      }
    }
  }
  if (rec->ring_depth > 0) {
    rec->amax_capacity = (epi == nms::kEpiArgmax) ? a->amax_capacity : 0;
    rec->pdl = (a->flags & NMS_FLAG_PDL) != 0;
    return NMS_OK;
  }
  rec->amax_capacity = (epi == nms::kEpiArgmax) ? a->amax_capacity : 0;
  rec->grid = dim3(grid);
  rec->block = dim3(nms::kGemvThreads);
  rec->smem = smem;
  rec->pdl = (a->flags & NMS_FLAG_PDL) != 0;
  return NMS_OK;
}

int prepare_attention(const nms_attention_args* a, LaunchRec* rec) {
  if (a == nullptr) return fail(NMS_ERR_VALUE, "args is null");
  if (!a->qkv || !a->k_cache || !a->v_cache || !a->rope || !a->pos || !a->y)
    return fail(NMS_ERR_VALUE, "null pointer argument");
  if (a->D != nms::kAttnD) return fail(NMS_ERR_NOT_IMPLEMENTED, "head_dim=%d (only %d is built)", a->D, nms::kAttnD);
  if (a->Hkv < 1 || a->Hq < a->Hkv || a->Hq % a->Hkv != 0)
    return fail(NMS_ERR_VALUE, "Hq=%d must be a positive multiple of Hkv=%d", a->Hq, a->Hkv);
  if (a->Hq / a->Hkv > nms::kAttnMaxGroup)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "GQA group %d > %d", a->Hq / a->Hkv, nms::kAttnMaxGroup);
  if (a->S_max < 1) return fail(NMS_ERR_VALUE, "S_max must be positive");
  if (a->rope_style != NMS_ROPE_INTERLEAVED && a->rope_style != NMS_ROPE_HALF)
    return fail(NMS_ERR_VALUE, "unknown rope_style %d", a->rope_style);
  if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16)) return fail(NMS_ERR_VALUE, "KV cache must be 16-byte aligned");
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  int splits = a->splits;
  if (splits <= 0) {
    splits = (dev->num_sms + a->Hkv - 1) / a->Hkv;
    if (splits > 16) splits = 16;
    if (splits < 1) splits = 1;
  }
  if (splits > 16) return fail(NMS_ERR_VALUE, "splits=%d > 16", splits);
  nms::AttnParams& p = rec->ap;
  p.qkv = static_cast<const __half*>(a->qkv);
  p.k_cache = static_cast<__half*>(a->k_cache);
  p.v_cache = static_cast<__half*>(a->v_cache);
  p.rope = static_cast<const __half*>(a->rope);
  p.q_norm = static_cast<const __half*>(a->q_norm);
  p.k_norm = static_cast<const __half*>(a->k_norm);
  p.pos = a->pos;
  p.y = static_cast<__half*>(a->y);
  p.norm_eps = a->norm_eps;
  p.scale = a->scale;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.S_max = a->S_max;
  p.rope_style = a->rope_style;
  p.splits = splits;
  rc = fill_next_prefetch(a->next_prefetch, a->next_prefetch_bytes, a->next_prefetch_head, p.next_pf,
                          p.next_pf_bytes, p.next_pf_head);
  if (rc) return rc;
  rec->kind = LaunchRec::kAttention;
  rec->grid = dim3(splits, a->Hkv);
  rec->block = dim3(nms::kAttnThreads);
  rec->cluster = dim3(splits, 1, 1);
  rec->smem = 0;
  rec->pdl = (a->flags & NMS_FLAG_PDL) != 0;
  return NMS_OK;
}

int prepare_embedding(const void* table, const int64_t* token, void* x, int64_t K, int64_t vocab, int32_t flags,
                      LaunchRec* rec) {
  if (!table || !token || !x) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (K <= 0 || K > (1 << 24) || vocab <= 0) return fail(NMS_ERR_VALUE, "bad sizes K=%lld vocab=%lld", (long long)K, (long long)vocab);
  rec->kind = LaunchRec::kEmbedding;
  rec->ep = EmbedParams{static_cast<const __half*>(table), token, static_cast<__half*>(x), (int)K, vocab};
  rec->grid = dim3((unsigned)((K + 255) / 256 < 64 ? (K + 255) / 256 : 64));
  rec->block = dim3(256);
  rec->smem = 0;
  rec->pdl = (flags & NMS_FLAG_PDL) != 0;
  return NMS_OK;
}

// ---------------------------------------------------------------------------
// Scratch of nms_gemv_argmax_noalloc_f16: the argmax partials of up to
// kNoAllocMaxCtas CTAs and the completion counter, in a file-scope device
// array instead of caller- or library-allocated memory.  Every GPU that loads
// this library holds it (8.5 KB) until the process exits.
constexpr int kNoAllocMaxCtas = 1024;
constexpr size_t kNoAllocValOff = 0;
constexpr size_t kNoAllocIdxOff = kNoAllocValOff + sizeof(float) * kNoAllocMaxCtas;
constexpr size_t kNoAllocCounterOff = kNoAllocIdxOff + sizeof(int32_t) * kNoAllocMaxCtas;
constexpr size_t kNoAllocBytes = 8448;
static_assert(kNoAllocCounterOff + sizeof(uint32_t) <= kNoAllocBytes, "no-alloc scratch layout");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (host code may not use the symbol itself as a pointer).
unsigned char* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NMS_ERR_VALUE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return NMS_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Prefill GEMM (nms_gemm.cuh): tile plan, workspace layout, tensor maps.
// ---------------------------------------------------------------------------
struct GemmPlan {
  int32_t m_tiles = 0, n_tiles = 0, bn = 0, splits = 1, stages = 0, atoms = 1, kblocks = 0;
  size_t smem = 0;
  int64_t total = 0;  // workspace bytes: xc [T, w_pad] fp16
};

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Clusters of `size` CTAs (one tile's k-splits) that can be resident at
// once with `smem` bytes of dynamic shared memory each; clusters are placed
// inside one GPC, so some sizes leave SMs unusable.  Cached per device.
int gemm_max_clusters(int size, size_t smem, int* out) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, int>, std::pair<size_t, int>>> cache;  // ((dev, size), (smem, n))
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& c : cache)
    if (c.first.first == dev && c.first.second == size && c.second.first == smem) {
      *out = c.second.second;
      return NMS_OK;
    }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(1, 1, (unsigned)size);
  cfg.blockDim = dim3(nms::kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeClusterDimension;
  a.val.clusterDim.x = 1;
  a.val.clusterDim.y = 1;
  a.val.clusterDim.z = (unsigned)size;
  cfg.attrs = &a;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, (const void*)nms::gemm_nm_kernel, &cfg);
  if (e != cudaSuccess) return fail_cuda(e, "cudaOccupancyMaxActiveClusters");
  cache.push_back({{dev, size}, {smem, n}});
  *out = n;
  return NMS_OK;
}

// One candidate shape of the prefill GEMM grid: token tiles of `bn`, `splits`
// k-splits per tile (a cluster), and its estimated time.  Measured on B200
// (per-CTA traces): the single producer and MMA-issuing threads pace a stage
// at ~0.45 us whatever its width, and the split-K epilogue (two cluster
// barriers, the distributed-shared-memory push and the reduction) costs
// ~1 us + 0.05 us per token column of the tile.
struct GemmCand {
  int32_t bn = 0, n_tiles = 0, atoms = 1, kblocks = 0, splits = 1, stages = 0;
  size_t smem = 0;
  int64_t ctas = 0, waves = 0, cost = 0;  // cost in units of 0.01 us
};

int gemm_candidate(int64_t T, int64_t w_pad, int32_t m_tiles, int32_t bn, int32_t splits_max, int num_sms,
                   size_t smem_max, GemmCand* c, bool* ok) {
  *ok = false;
  c->bn = bn;
  c->n_tiles = (int32_t)((T + bn - 1) / bn);
  c->atoms = bn <= 64 ? 2 : 1;
  c->kblocks = (int32_t)((w_pad / nms::kGemmBK + c->atoms - 1) / c->atoms);
  const size_t stage = ((size_t)nms::kGemmBM * 128 + (size_t)bn * 128) * c->atoms;
  const size_t avail = smem_max > 1024 ? smem_max - 1024 : 0;
  c->stages = (int32_t)std::min<size_t>(nms::kGemmMaxStages, avail / stage);
  if (c->stages < 2) return NMS_OK;
  c->smem = 1024 + (size_t)c->stages * stage;
  const int64_t tiles = (int64_t)m_tiles * c->n_tiles;
  c->splits = (int32_t)std::max<int64_t>(1, std::min<int64_t>(splits_max, c->kblocks));
  // Keep every tile's cluster resident in one wave: shrink the split count
  // until the GPCs hold `tiles` clusters of that size.
  while (c->splits > 1) {
    int fit = 0;
    int rc = gemm_max_clusters(c->splits, c->smem, &fit);
    if (rc) return rc;
    if (fit >= tiles) break;
    --c->splits;
  }
  // Epilogue staging reuses the ring: fp16 output rows, after the split-K
  // receive buffer (splits x 128 rows x (owned columns + 4) fp32) when split.
  const int64_t ncl = (bn / 16 + c->splits - 1) / c->splits * 16;
  const size_t staging = c->splits > 1
                             ? (size_t)c->splits * nms::kGemmBM * (ncl + 4) * 4 + (size_t)ncl * nms::kGemmOutPitch * 2
                             : (size_t)bn * nms::kGemmOutPitch * 2;
  if (staging > (size_t)c->stages * stage) return NMS_OK;
  c->ctas = tiles * c->splits;
  c->waves = (c->ctas + num_sms - 1) / num_sms;  // one CTA per SM (shared memory)
  const int64_t per_cta = (c->kblocks + c->splits - 1) / c->splits * 45 + (c->splits > 1 ? 100 + 5 * bn : 0);
  c->cost = c->waves * per_cta;
  *ok = true;
  return NMS_OK;
}

// Tokens are split into ceil(T / 256) equal tiles (UMMA N <= 256, a multiple
// of 16); rows of h into 128-row tiles.  The default plan splits the
// compressed width when the tiles leave SMs idle (a cluster of up to 8 CTAs
// per tile: every weight byte is still loaded once), and halves the token
// tiles (down to 32) only while that still fills less than half the SMs.
// Other candidates -- each halving of the token tile, unsplit or split -- are
// costed with the model above, and one replaces the default only if it is
// estimated at least 10% faster (ties: fewer waves, then more CTAs).  Token
// tiles of <= 64 take two 64-column atoms per stage, so one barrier round
// trip of the producer and MMA threads feeds 8 MMAs instead of 4.
int gemm_plan(int64_t T, int64_t w_pad, int64_t h, int num_sms, size_t smem_max, GemmPlan* g) {
  g->m_tiles = (int32_t)((h + nms::kGemmBM - 1) / nms::kGemmBM);
  const int32_t n0 = (int32_t)((T + nms::kGemmMaxBN - 1) / nms::kGemmMaxBN);
  const int32_t bn0 = (int32_t)std::max<int64_t>(16, round_up((T + n0 - 1) / n0, 16));
  auto smax = [&](int32_t bn) -> int32_t {
    const int64_t tiles = (int64_t)g->m_tiles * ((T + bn - 1) / bn);
    return tiles < num_sms ? (int32_t)std::min<int64_t>(8, num_sms / tiles) : 1;
  };
  // The default plan.
  int32_t bn_def = bn0;
  while (bn_def >= 64 && (int64_t)g->m_tiles * ((T + bn_def - 1) / bn_def) * smax(bn_def) * 2 <= num_sms)
    bn_def = (int32_t)round_up(bn_def / 2, 16);
  GemmCand best;
  bool ok = false;
  int rc = gemm_candidate(T, w_pad, g->m_tiles, bn_def, smax(bn_def), num_sms, smem_max, &best, &ok);
  if (rc) return rc;
  if (!ok) return fail(NMS_ERR_NOT_IMPLEMENTED, "gemm: no grid fits %zu B of shared memory", smem_max);
  const int64_t def_cost = best.cost;
  GemmCand alt;
  bool have_alt = false;
  for (int32_t bn = bn0;; bn = (int32_t)round_up(bn / 2, 16)) {
    for (int32_t sm : {1, smax(bn)}) {
      GemmCand c;
      rc = gemm_candidate(T, w_pad, g->m_tiles, bn, sm, num_sms, smem_max, &c, &ok);
      if (rc) return rc;
      if (!ok || (c.bn == best.bn && c.splits == best.splits)) continue;
      if (!have_alt || c.cost < alt.cost ||
          (c.cost == alt.cost && (c.waves < alt.waves || (c.waves == alt.waves && c.ctas > alt.ctas)))) {
        alt = c;
        have_alt = true;
      }
    }
    if (bn < 64) break;
  }
  if (have_alt && alt.cost * 10 <= def_cost * 9) best = alt;
  g->bn = best.bn;
  g->n_tiles = best.n_tiles;
  g->atoms = best.atoms;
  g->kblocks = best.kblocks;
  g->splits = best.splits;
  g->stages = best.stages;
  g->smem = best.smem;
  g->total = round_up(T * w_pad * 2, 256);
  return NMS_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled_fn(EncodeTiledFn* out) {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || p == nullptr)
      return fail(NMS_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return NMS_OK;
}

// 2-D fp16 tensor map over a row-major [rows, cols] matrix: boxes of
// 64 columns (128 bytes) x box_rows rows, 128-byte swizzle, zero fill outside.
int encode_k_major(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int32_t box_rows) {
  EncodeTiledFn fn = nullptr;
  int rc = encode_tiled_fn(&fn);
  if (rc) return rc;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)nms::kGemmBK, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NMS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NMS_OK;
}

int gemm_check_shape(int64_t T, int64_t K, int64_t w, int64_t w_pad, int64_t h, int32_t block_width,
                     int32_t vec_width) {
  if (T <= 0 || T > (1 << 24)) return fail(NMS_ERR_VALUE, "T=%lld must be in [1, 2^24]", (long long)T);
  if (h <= 0 || h > (1ll << 30)) return fail(NMS_ERR_VALUE, "h=%lld out of range", (long long)h);
  if (block_width <= 0 || vec_width <= 0) return fail(NMS_ERR_VALUE, "N and M must be positive");
  if (block_width > vec_width || vec_width > 256)
    return fail(NMS_ERR_VALUE, "N=%d, M=%d: need N <= M <= 256", block_width, vec_width);
  if (w <= 0 || w % block_width != 0) return fail(NMS_ERR_VALUE, "w=%lld must be divisible by N=%d", (long long)w, block_width);
  if (K != (w / block_width) * vec_width)
    return fail(NMS_ERR_VALUE, "K=%lld must equal (w/N)*M=%lld", (long long)K, (long long)((w / block_width) * vec_width));
  if (K > (1ll << 30)) return fail(NMS_ERR_VALUE, "K=%lld out of range", (long long)K);
  if (w_pad != nms_packed_row_stride(w))
    return fail(NMS_ERR_VALUE, "w_pad=%lld must be %lld", (long long)w_pad, (long long)nms_packed_row_stride(w));
  return NMS_OK;
}

struct nms_plan {
  std::vector<LaunchRec> recs;
};

struct nms_step {
  int device = 0;
  int nstages = 0;
  int grid = 0;
  size_t smem = 0;
  int depth = 0;            // weight-ring depth (selects the kernel instantiation)
  std::vector<nms::StepGemv> gemvs;    // host copy of the device GEMV stage table
  std::vector<int32_t> gemv_of_stage;  // stage -> GEMV ordinal (-1: attention)
  void* dev_mem = nullptr;  // stage tables | barrier words | attention partials | head counters
  size_t bar_bytes = 0;     // barrier words at params.bar_count (arrivals, exits)
  size_t cnt_bytes = 0;     // per-head attention arrival counters at params.attn_count
  bool flow = false;        // dataflow kernel (decode_flow_kernel) instead of the barrier kernel
  nms::FlowParams fparams;  // flow: kernel parameters (tables and words live in dev_mem)
  nms::StepParams params;
};

extern "C" {

int nms_abi_version(void) { return NMS_ABI_VERSION; }

#ifndef NMS_SOURCE_HASH
#define NMS_SOURCE_HASH "unknown"
#endif
const char* nms_source_hash(void) { return NMS_SOURCE_HASH; }

const char* nms_last_error(void) { return g_last_error.c_str(); }

const char* nms_status_name(int status) {
  switch (status) {
    case NMS_OK: return "NMS_OK";
    case NMS_ERR_VALUE: return "NMS_ERR_VALUE";
    case NMS_ERR_TYPE: return "NMS_ERR_TYPE";
    case NMS_ERR_NOT_IMPLEMENTED: return "NMS_ERR_NOT_IMPLEMENTED";
    case NMS_ERR_CUDA: return "NMS_ERR_CUDA";
    case NMS_ERR_DEVICE: return "NMS_ERR_DEVICE";
    default: return "NMS_ERR_UNKNOWN";
  }
}

int nms_num_sms(int* out) {
  if (out == nullptr) return fail(NMS_ERR_VALUE, "out is null");
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  *out = dev->num_sms;
  return NMS_OK;
}

int nms_device_error(int* code_out, int clear) {
  if (code_out == nullptr) return fail(NMS_ERR_VALUE, "code_out is null");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, nms::g_device_error, sizeof(int));
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemcpyFromSymbol(device error)");
  *code_out = v;
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(nms::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemcpyToSymbol(device error)");
  }
  return NMS_OK;
}

int nms_device_error_set(int code) {
  if (code <= 0) return fail(NMS_ERR_VALUE, "code must be positive (got %d); clear with nms_device_error", code);
  cudaError_t e = cudaMemcpyToSymbol(nms::g_device_error, &code, sizeof(int));
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemcpyToSymbol(device error)");
  return NMS_OK;
}

static int gemv_ref_launch(const void* vec, const void* mat_data, const void* mat_index, void* out, int64_t K,
                           int64_t w, int64_t h, int32_t block_width, int32_t vec_width, void* stream, bool rowwise) {
  if (!vec || !mat_data || !mat_index || !out) return fail(NMS_ERR_VALUE, "null pointer argument");
  int rc = check_nm(K, w, block_width, vec_width);
  if (rc) return rc;
  if (h <= 0 || h % 128 != 0) return fail(NMS_ERR_VALUE, "h must be divisible by 128 (got %lld)", (long long)h);
  if (h > (1 << 28)) return fail(NMS_ERR_VALUE, "h=%lld too large", (long long)h);
  if (!aligned(mat_data, 32)) return fail(NMS_ERR_VALUE, "mat_data must be 32-byte aligned");
  if (rowwise && !aligned(mat_index, 16)) return fail(NMS_ERR_VALUE, "per-row mat_index must be 16-byte aligned");
  const DeviceInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  constexpr int LR = 8, RB = 16 * LR;
  const int64_t nblocks = h / RB;
  int cs = (int)((2 * dev->num_sms + nblocks - 1) / nblocks);
  if (cs > 8) cs = 8;
  const int64_t max_cs_by_width = w / 256 > 0 ? w / 256 : 1;
  if (cs > max_cs_by_width) cs = (int)max_cs_by_width;
  if (cs < 1) cs = 1;
  const int64_t jchunk = (w + cs - 1) / cs;
  LaunchRec rec;
  nms::GemvRefParams& p = rec.rp;
  p.vec = static_cast<const __half*>(vec);
  p.mat_data = static_cast<const __half*>(mat_data);
  p.mat_index = static_cast<const uint8_t*>(mat_index);
  p.out = static_cast<__half*>(out);
  p.K = (int32_t)K;
  p.w = (int32_t)w;
  p.h = (int32_t)h;
  p.n = block_width;
  p.m = vec_width;
  p.jchunk = (int32_t)jchunk;
  p.cs = cs;
  rec.kind = LaunchRec::kGemvRef;
  rec.rowwise = rowwise;
  rec.smem = nms::align_up_sz((size_t)(rowwise ? K + 256 : jchunk) * 2, 16) + (size_t)(nms::kGemvWarps + 1) * RB * 4;
  if (rec.smem > dev->max_smem_optin)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "%s too large for one CTA slice", rowwise ? "K" : "w");
  rec.grid = dim3((unsigned)nblocks, (unsigned)cs);
  rec.block = dim3(nms::kGemvThreads);
  rec.cluster = dim3(1, (unsigned)cs, 1);
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_gemv_f16(const void* vec, const void* mat_data, const void* mat_index, void* out, int64_t K, int64_t w,
                 int64_t h, int32_t block_width, int32_t vec_width, void* stream) {
  return gemv_ref_launch(vec, mat_data, mat_index, out, K, w, h, block_width, vec_width, stream, false);
}

int nms_gemv_rowwise_f16(const void* vec, const void* mat_data, const void* mat_index, void* out, int64_t K,
                         int64_t w, int64_t h, int32_t block_width, int32_t vec_width, void* stream) {
  return gemv_ref_launch(vec, mat_data, mat_index, out, K, w, h, block_width, vec_width, stream, true);
}

int64_t nms_packed_row_stride(int64_t w) {
  if (w <= 0) return 0;
  return (w + 63) / 64 * 64;
}

static int pack_common(const void* src, void* dst, int64_t w, int64_t h, int64_t w_pad, void* stream, bool pack) {
  if (!src || !dst) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (w <= 0 || h <= 0 || w_pad < w)
    return fail(NMS_ERR_VALUE, "bad sizes w=%lld h=%lld w_pad=%lld", (long long)w, (long long)h, (long long)w_pad);
  if (w_pad > (1 << 26) || h > (1 << 26)) return fail(NMS_ERR_VALUE, "sizes too large");
  LaunchRec rec;
  rec.kind = pack ? LaunchRec::kPack : LaunchRec::kUnpack;
  rec.pk.src = static_cast<const __half*>(src);
  rec.pk.dst = static_cast<__half*>(dst);
  rec.pk.w = (int)w;
  rec.pk.h = (int)h;
  rec.pk.w_pad = (int)w_pad;
  rec.grid = dim3((unsigned)(((pack ? w_pad : w) + 31) / 32), (unsigned)((h + 31) / 32));
  rec.block = dim3(32, 8);
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_pack_f16(const void* mat_data, void* packed, int64_t w, int64_t h, int64_t w_pad, void* stream) {
  return pack_common(mat_data, packed, w, h, w_pad, stream, true);
}

int nms_unpack_f16(const void* packed, void* mat_data, int64_t w, int64_t h, int64_t w_pad, void* stream) {
  return pack_common(packed, mat_data, w, h, w_pad, stream, false);
}

int nms_gemv_packed_f16(const void* vec, const void* packed, const void* mat_index, void* out, int64_t K, int64_t w,
                        int64_t w_pad, int64_t h, int32_t block_width, int32_t vec_width, void* stream) {
  if (!vec || !packed || !mat_index || !out) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (h <= 0) return fail(NMS_ERR_VALUE, "h must be positive");
  nms_gemv_fused_args a;
  memset(&a, 0, sizeof(a));
  a.seg[0].packed = packed;
  a.seg[0].mat_index = mat_index;
  a.seg[0].rows = h;
  a.nseg = 1;
  a.epilogue = NMS_EPI_STORE;
  a.prologue = NMS_PRO_PLAIN;
  a.K = K;
  a.w = w;
  a.w_pad = w_pad;
  a.block_width = block_width;
  a.vec_width = vec_width;
  a.x = vec;
  a.out = out;
  LaunchRec rec;
  int rc = prepare_gemv(&a, &rec);
  if (rc) return rc;
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_gemv_fused_f16(const nms_gemv_fused_args* args, void* stream) {
  LaunchRec rec;
  int rc = prepare_gemv(args, &rec);
  if (rc) return rc;
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_attention_decode_f16(const nms_attention_args* args, void* stream) {
  LaunchRec rec;
  int rc = prepare_attention(args, &rec);
  if (rc) return rc;
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_embedding_f16(const void* table, const int64_t* token, void* x, int64_t K, int64_t vocab, int32_t flags,
                      void* stream) {
  LaunchRec rec;
  int rc = prepare_embedding(table, token, x, K, vocab, flags, &rec);
  if (rc) return rc;
  return launch_rec(rec, static_cast<cudaStream_t>(stream));
}

int nms_gemv_argmax_noalloc_f16(const void* x, const void* x2, const void* norm_weight, float eps,
                                const void* head_weight, int64_t vocab, int64_t K, void* logits, int64_t* token_out,
                                void* stream) {
  if (!x || !head_weight || !logits || !token_out) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (vocab <= 0 || vocab > (1 << 30)) return fail(NMS_ERR_VALUE, "vocab=%lld out of range", (long long)vocab);
  if (K <= 0 || K % 64 != 0) return fail(NMS_ERR_VALUE, "K=%lld must be a positive multiple of 64", (long long)K);
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  // One CTA per (up to) two SMs' worth of rows; the scratch holds
  // kNoAllocMaxCtas partials, so larger launches are refused.
  const int L = pick_lanes_per_row(K);
  const int64_t row_groups = (vocab + (32 / L) - 1) / (32 / L);
  const int64_t grid = row_groups < (int64_t)dev->num_sms * kGemvCtasPerSm ? row_groups
                                                                          : (int64_t)dev->num_sms * kGemvCtasPerSm;
  if (grid > kNoAllocMaxCtas)
    return fail(NMS_ERR_VALUE, "launch needs %lld argmax partials; the static scratch holds %d", (long long)grid,
                kNoAllocMaxCtas);
  unsigned char* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  nms_gemv_fused_args a;
  memset(&a, 0, sizeof(a));
  a.seg[0].packed = head_weight;
  a.seg[0].rows = vocab;
  a.nseg = 1;
  a.epilogue = NMS_EPI_ARGMAX;
  a.prologue = norm_weight ? NMS_PRO_RESID_RMSNORM : NMS_PRO_PLAIN;
  a.flags = NMS_FLAG_DENSE;
  a.K = K;
  a.w = K;
  a.w_pad = K;
  a.x = x;
  a.x2 = norm_weight ? x2 : nullptr;
  a.norm_weight = norm_weight;
  a.eps = eps;
  a.out = logits;
  a.amax_val = reinterpret_cast<float*>(scratch + kNoAllocValOff);
  a.amax_idx = reinterpret_cast<int32_t*>(scratch + kNoAllocIdxOff);
  a.amax_counter = reinterpret_cast<uint32_t*>(scratch + kNoAllocCounterOff);
  a.token_out = token_out;
  a.amax_capacity = kNoAllocMaxCtas;
  a.grid = (int32_t)grid;
  LaunchRec rec;
  rc = prepare_gemv(&a, &rec);
  if (rc) return rc;
  // The counter must start at zero; an earlier call leaves it at zero when it
  // completes, and this clears it after an aborted one.
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(scratch + kNoAllocCounterOff, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(no-alloc counter)");
  return launch_rec(rec, st);
}

int nms_plan_create(nms_plan** out) {
  if (out == nullptr) return fail(NMS_ERR_VALUE, "out is null");
  *out = new (std::nothrow) nms_plan();
  if (*out == nullptr) return fail(NMS_ERR_CUDA, "out of host memory");
  return NMS_OK;
}

int nms_plan_destroy(nms_plan* plan) {
  delete plan;
  return NMS_OK;
}

int nms_plan_add_gemv(nms_plan* plan, const nms_gemv_fused_args* args) {
  if (plan == nullptr) return fail(NMS_ERR_VALUE, "plan is null");
  LaunchRec rec;
  int rc = prepare_gemv(args, &rec);
  if (rc) return rc;
  plan->recs.push_back(rec);
  return NMS_OK;
}

int nms_plan_add_attention(nms_plan* plan, const nms_attention_args* args) {
  if (plan == nullptr) return fail(NMS_ERR_VALUE, "plan is null");
  LaunchRec rec;
  int rc = prepare_attention(args, &rec);
  if (rc) return rc;
  plan->recs.push_back(rec);
  return NMS_OK;
}

int nms_plan_add_embedding(nms_plan* plan, const void* table, const int64_t* token, void* x, int64_t K, int64_t vocab,
                           int32_t flags) {
  if (plan == nullptr) return fail(NMS_ERR_VALUE, "plan is null");
  LaunchRec rec;
  int rc = prepare_embedding(table, token, x, K, vocab, flags, &rec);
  if (rc) return rc;
  plan->recs.push_back(rec);
  return NMS_OK;
}

int nms_plan_size(const nms_plan* plan, int32_t* out) {
  if (plan == nullptr || out == nullptr) return fail(NMS_ERR_VALUE, "null argument");
  *out = (int32_t)plan->recs.size();
  return NMS_OK;
}

int nms_step_create(const nms_plan* plan, const int32_t* records, int32_t nrecords, nms_step** out) {
  if (plan == nullptr || out == nullptr || records == nullptr) return fail(NMS_ERR_VALUE, "null argument");
  const int32_t n = (int32_t)plan->recs.size();
  if (nrecords < 1) return fail(NMS_ERR_VALUE, "no records");
  for (int32_t k = 0; k < nrecords; ++k)
    if (records[k] < 0 || records[k] >= n) return fail(NMS_ERR_VALUE, "record %d outside plan of %d", records[k], n);
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int grid = dev->num_sms;
  std::vector<int32_t> kinds;
  std::vector<nms::StepGemv> gemvs;
  std::vector<nms::ProdDesc> descs;
  std::vector<nms::AttnParams> attns;
  size_t act = sizeof(nms::StepAttnSmem);
  int max_units = 0, max_hkv = 0;
  const int64_t* pos_ptr = nullptr;
  for (int32_t k = 0; k < nrecords; ++k) {
    const int32_t i = records[k];
    const LaunchRec& r = plan->recs[i];
    if (r.kind == LaunchRec::kGemvPacked) {
      nms::StepGemv sg;
      memset(&sg, 0, sizeof(sg));
      sg.g = r.gp;
      sg.lanes = nms::ring_lanes(sg.g.w_pad);
      sg.tp_send = sg.tp_recv = -1;
      const int RG = 32 / sg.lanes;
      sg.g.row_groups = (sg.g.rows_total + RG - 1) / RG;
      if (sg.g.epilogue == nms::kEpiArgmax && (sg.g.amax_val == nullptr || grid > r.amax_capacity))
        return fail(NMS_ERR_VALUE, "record %d: argmax scratch holds %d partials, the step needs %d", i,
                    r.amax_capacity, grid);
      const bool paired = sg.g.mode == nms::kModePaired;
      const int nsegx = paired ? 2 : sg.g.nseg;
      const int max_vrows = (paired ? 2 : 1) * ((sg.g.row_groups + grid - 1) / grid) * RG;
      const size_t need = nms::step_gemv_smem_bytes(sg.g.K, sg.g.w, sg.g.w_pad, nsegx, max_vrows,
                                                    sg.g.prologue == nms::kProResidNorm);
      if (need > act) act = need;
      nms::ProdDesc pd;
      memset(&pd, 0, sizeof(pd));
      for (int k = 0; k < sg.g.nseg; ++k) {
        pd.w[k] = sg.g.seg[k].w;
        pd.row_start[k] = sg.g.seg[k].row_start;
      }
      pd.rows_total = sg.g.rows_total;
      pd.row_groups = sg.g.row_groups;
      pd.w_pad = sg.g.w_pad;
      pd.nseg = (int16_t)sg.g.nseg;
      pd.paired = paired ? 1 : 0;
      pd.lanes = (int8_t)sg.lanes;
      kinds.push_back(nms::kStageGemv);
      gemvs.push_back(sg);
      descs.push_back(pd);
    } else if (r.kind == LaunchRec::kAttention) {
      if (r.ap.splits > nms::kMaxSplits)
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: %d attention splits (max %d)", i, r.ap.splits, nms::kMaxSplits);
      const int units = r.ap.Hkv * r.ap.splits;
      if (pos_ptr == nullptr) pos_ptr = r.ap.pos;
      if (r.ap.pos != pos_ptr) return fail(NMS_ERR_VALUE, "record %d: attention stages must share one position", i);
      if (units > max_units) max_units = units;
      if (r.ap.Hkv > max_hkv) max_hkv = r.ap.Hkv;
      kinds.push_back(nms::kStageAttn);
      attns.push_back(r.ap);
    } else {
      return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: only GEMV and attention launches run in a persistent step", i);
    }
  }
  // Shared memory: [rings: 32 warps x D items][working set][stream descriptors][stage kinds].
  act = nms::align_up_sz(act, 128);
  const size_t tail_bytes = descs.size() * sizeof(nms::ProdDesc) + nms::align_up_sz(kinds.size() * 4, 16);
  const size_t ring_unit = (size_t)nms::kStepWarps * nms::kRingItemBytes;
  int depth = 0;
  for (int d : {nms::kStepDepthHi, nms::kStepDepthLo})
    if (depth == 0 && (size_t)d * ring_unit + act + tail_bytes <= dev->step_smem_max) depth = d;
  if (depth == 0)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "persistent step: a %zu-byte working set leaves no room for the weight rings",
                act);
  const size_t ring_bytes = (size_t)depth * ring_unit;
  const size_t smem = ring_bytes + act + tail_bytes;

  const size_t kind_off = 0;
  const size_t gemv_off = nms::align_up_sz(kind_off + kinds.size() * 4, 256);
  const size_t desc_off = nms::align_up_sz(gemv_off + gemvs.size() * sizeof(nms::StepGemv), 256);
  const size_t attn_off = nms::align_up_sz(desc_off + descs.size() * sizeof(nms::ProdDesc), 256);
  const size_t bar_off = nms::align_up_sz(attn_off + attns.size() * sizeof(nms::AttnParams), 256);
  const size_t part_off = bar_off + 256;
  const size_t part_bytes = (size_t)max_units * nms::kAttnMaxGroup * (nms::kAttnD + 2) * sizeof(float);
  const size_t cnt_off = nms::align_up_sz(part_off + part_bytes, 256);
  const size_t total = cnt_off + nms::align_up_sz((size_t)(max_hkv > 0 ? max_hkv : 1) * sizeof(unsigned), 256);
  nms_step* st = new (std::nothrow) nms_step();
  if (st == nullptr) return fail(NMS_ERR_CUDA, "out of host memory");
  cudaError_t e = cudaGetDevice(&st->device);
  if (e == cudaSuccess) e = cudaMalloc(&st->dev_mem, total);
  if (e == cudaSuccess) e = cudaMemset(st->dev_mem, 0, total);
  unsigned char* base = static_cast<unsigned char*>(st->dev_mem);
  if (e == cudaSuccess) e = cudaMemcpy(base + kind_off, kinds.data(), kinds.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !gemvs.empty())
    e = cudaMemcpy(base + gemv_off, gemvs.data(), gemvs.size() * sizeof(nms::StepGemv), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !descs.empty())
    e = cudaMemcpy(base + desc_off, descs.data(), descs.size() * sizeof(nms::ProdDesc), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !attns.empty())
    e = cudaMemcpy(base + attn_off, attns.data(), attns.size() * sizeof(nms::AttnParams), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (st->dev_mem) cudaFree(st->dev_mem);
    delete st;
    return fail_cuda(e, "persistent step set-up");
  }
  st->nstages = (int)kinds.size();
  st->grid = grid;
  st->smem = smem;
  st->depth = depth;
  nms::StepParams& P = st->params;
  memset(&P, 0, sizeof(P));
  P.kind = reinterpret_cast<const int32_t*>(base + kind_off);
  P.gemv = reinterpret_cast<const nms::StepGemv*>(base + gemv_off);
  P.desc = reinterpret_cast<const nms::ProdDesc*>(base + desc_off);
  P.attn = reinterpret_cast<const nms::AttnParams*>(base + attn_off);
  P.nstages = st->nstages;
  P.ngemv = (int32_t)gemvs.size();
  P.nattn = (int32_t)attns.size();
  P.ring_bytes = (int32_t)ring_bytes;
  P.act_bytes = (int32_t)act;
  P.bar_count = reinterpret_cast<unsigned*>(base + bar_off);
  P.bar_exit = reinterpret_cast<unsigned*>(base + bar_off + 128);
  P.attn_part = reinterpret_cast<float*>(base + part_off);
  P.attn_count = reinterpret_cast<unsigned*>(base + cnt_off);
  P.trace = nullptr;
  P.pos = pos_ptr;
  P.tp_world = 1;
  st->bar_bytes = 192;  // bar_count at +0, bar_exit at +128 (the head's local winner follows at +192)
  st->cnt_bytes = total - cnt_off;
  st->gemvs = gemvs;
  st->gemv_of_stage.assign(kinds.size(), -1);
  for (size_t k = 0, g = 0; k < kinds.size(); ++k)
    if (kinds[k] == nms::kStageGemv) st->gemv_of_stage[k] = (int32_t)g++;
  *out = st;
  return NMS_OK;
}

// ---------------------------------------------------------------------------
// Dataflow persistent step (decode_flow_kernel).  The routing of every
// stage's output is derived from the plan records by pointer identity:
//   * a residual + RMSNorm GEMV N (x, x2, norm, resid_out) makes the GEMV
//     whose output is x2 a residual producer: it reads the residual words
//     that stand for x, writes resid_new (standing for N's resid_out), its
//     sum-of-squares partials, and scatters resid_new into N's compressed
//     inputs (one inverse table per mask segment of N);
//   * a plain GEMV N reads the output of the attention stage or SwiGLU GEMV
//     that writes its x, scattered the same way;
//   * an attention stage reads the words of the GEMV that writes its qkv;
//   * the first stage may read the embedding row (x_token) and gathers it
//     by mask itself.
// Anything else is refused with NMS_ERR_NOT_IMPLEMENTED (the caller then
// uses nms_step_create).  Device memory, one block: [static tables (inverse
// maps, mask-gathered norm weights) | stage tables, words, partials].
// ---------------------------------------------------------------------------
}  // extern "C"

namespace {

struct FlowArena {
  size_t static_end = 0, end = 0;
  std::vector<unsigned char> init;  // host image of the static region
  size_t take_static(size_t bytes) {
    const size_t off = nms::align_up_sz(static_end, 256);
    static_end = off + bytes;
    init.resize(static_end, 0);
    return off;
  }
  size_t take_dyn(size_t bytes) {
    const size_t off = nms::align_up_sz(end, 256);
    end = off + bytes;
    return off;
  }
};

enum : int { kOwnNone = 0, kOwnGemv = 1, kOwnAttn = 2 };
struct FlowOwner {
  int kind = kOwnNone, index = -1;
};

// Offsets stand in for device pointers until the block is allocated; the
// top bit marks an offset into the dynamic region, +1 keeps offset 0 apart
// from nullptr.
constexpr uintptr_t kFlowDynBit = (uintptr_t)1 << 62;
template <typename T>
T* flow_off(size_t off, bool dynamic) {
  return reinterpret_cast<T*>((uintptr_t)(off + 1) | (dynamic ? kFlowDynBit : 0));
}

int read_mask(const nms::GemvParams& g, int sx, std::vector<uint8_t>* idx) {
  idx->resize((size_t)g.w);
  cudaError_t e = cudaMemcpy(idx->data(), g.seg[sx].idx, (size_t)g.w, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? NMS_OK : fail_cuda(e, "reading mat_index");
}

}  // namespace

extern "C" {

int nms_step_create_flow(const nms_plan* plan, const int32_t* records, int32_t nrecords, nms_step** out) {
  if (plan == nullptr || out == nullptr || records == nullptr) return fail(NMS_ERR_VALUE, "null argument");
  const int32_t n = (int32_t)plan->recs.size();
  if (nrecords < 1) return fail(NMS_ERR_VALUE, "no records");
  for (int32_t k = 0; k < nrecords; ++k)
    if (records[k] < 0 || records[k] >= n) return fail(NMS_ERR_VALUE, "record %d outside plan of %d", records[k], n);
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int grid = dev->num_sms;
  constexpr int NT = nms::kStepThreads;

  std::vector<int32_t> kinds;
  std::vector<nms::FlowGemv> fg;
  std::vector<nms::ProdDesc> descs;
  std::vector<nms::FlowAttn> fa;
  FlowArena ar;
  std::map<const void*, FlowOwner> out_owner;
  std::map<const void*, uint32_t*> resid_of;  // plain residual vector -> words standing for it
  std::vector<uint32_t*> natural_of_gemv;      // natural-order output words of a GEMV (nullptr: none)
  std::vector<uint32_t*> natural_of_attn;
  size_t act = sizeof(nms::StepAttnSmem);
  const int64_t* pos_ptr = nullptr;
  int nstage_counter = 0;  // completion counters, one per stage (offsets patched once the block exists)

  for (int32_t k = 0; k < nrecords; ++k) {
    const int32_t i = records[k];
    const LaunchRec& r = plan->recs[i];
    if (r.kind == LaunchRec::kGemvPacked) {
      const int gi = (int)fg.size();
      nms::FlowGemv f;
      memset(&f, 0, sizeof(f));
      nms::StepGemv& sg = f.sg;
      sg.g = r.gp;
      sg.lanes = nms::ring_lanes(sg.g.w_pad);
      sg.tp_send = sg.tp_recv = -1;
      const int RG = 32 / sg.lanes;
      sg.g.row_groups = (sg.g.rows_total + RG - 1) / RG;
      const nms::GemvParams& g = sg.g;
      if (g.epilogue == nms::kEpiArgmax && (g.amax_val == nullptr || grid > r.amax_capacity))
        return fail(NMS_ERR_VALUE, "record %d: argmax scratch holds %d partials, the step needs %d", i,
                    r.amax_capacity, grid);
      const bool paired = g.mode == nms::kModePaired;
      const int nsegx = paired ? 2 : g.nseg;
      const bool dense = g.seg[0].idx == nullptr;
      const bool norm = g.prologue == nms::kProResidNorm;
      const int max_vrows = (paired ? 2 : 1) * ((g.row_groups + grid - 1) / grid) * RG;
      f.out_mode = -1;
      f.in_mode = nms::kFlowInTagged;
      f.done_out = flow_off<unsigned>((size_t)(nstage_counter++) * 4, true);  // offset into the counter block, patched below
      if (dense && (g.w != g.K || g.w_pad != g.K))
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: dense stage with w != K", i);
      // This stage's compressed inputs and the producer's scatter targets;
      // `natural`: the producer's natural-order words (allocated here when a
      // dense input needs them).
      auto route_inputs = [&](int prod_kind, int prod_index) -> int {
        uint32_t*& natural = prod_kind == kOwnGemv ? natural_of_gemv[prod_index] : natural_of_attn[prod_index];
        for (int sx = 0; sx < nsegx; ++sx) {
          if (dense) {
            if (natural == nullptr) natural = flow_off<uint32_t>(ar.take_dyn((size_t)g.K * 4), true);
            f.xc_in[sx] = natural;
            continue;
          }
          std::vector<uint8_t> idx;
          int rc2 = read_mask(g, sx, &idx);
          if (rc2) return rc2;
          const size_t inv_off = ar.take_static((size_t)g.K * 4);
          int32_t* inv = reinterpret_cast<int32_t*>(ar.init.data() + inv_off);
          for (int c = 0; c < g.K; ++c) inv[c] = -1;
          for (int j = 0; j < g.w; ++j) {
            const int col = (j / g.n) * g.m + (int)idx[j];
            if ((int)idx[j] >= g.m || col >= g.K || inv[col] != -1)
              return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: mask segment %d is not an N:M selection", i, sx);
            inv[col] = j;
          }
          uint32_t* xc = flow_off<uint32_t>(ar.take_dyn((size_t)g.w_pad * 4), true);
          f.xc_in[sx] = xc;
          const int32_t* invp = flow_off<const int32_t>(inv_off, false);
          if (prod_kind == kOwnGemv) {
            nms::FlowGemv& P = fg[prod_index];
            if (P.nscat >= nms::kFlowMaxScat)
              return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: too many scatter targets", i);
            P.scat_dst[P.nscat] = xc;
            P.scat_inv[P.nscat] = invp;
            ++P.nscat;
          } else {
            nms::FlowAttn& A = fa[prod_index];
            if (A.y_dst != nullptr)
              return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: attention output feeds two masks", i);
            A.y_dst = xc;
            A.y_inv = invp;
          }
        }
        return NMS_OK;
      };
      if (g.x_token != nullptr) {
        if (k != 0) return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: only the first stage may read the embedding", i);
        f.in_mode = nms::kFlowInGather;
        if (g.resid_out != nullptr) {
          f.gather_resid = flow_off<uint32_t>(ar.take_dyn((size_t)g.K * 4), true);
          resid_of[g.resid_out] = f.gather_resid;
        }
      } else if (norm) {
        auto it = out_owner.find(g.x2);
        auto rx = resid_of.find(g.x);
        if (g.x2 == nullptr || it == out_owner.end() || it->second.kind != kOwnGemv || rx == resid_of.end())
          return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: residual inputs are not produced inside the step", i);
        nms::FlowGemv& P = fg[it->second.index];
        if (P.out_mode != -1 || P.sg.g.epilogue != nms::kEpiStore || P.sg.g.mode == nms::kModePaired ||
            P.sg.g.rows_total != g.K)
          return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: residual producer is not a plain %d-row GEMV", i, g.K);
        P.out_mode = nms::kFlowOutResid;
        P.resid_old = rx->second;
        uint32_t* words = flow_off<uint32_t>(ar.take_dyn((size_t)g.K * 4), true);
        natural_of_gemv[it->second.index] = words;
        if (g.resid_out != nullptr) resid_of[g.resid_out] = words;
        P.ssq_out = flow_off<unsigned long long>(ar.take_dyn((size_t)grid * 8), true);
        f.ssq_in = P.ssq_out;
        f.done_in = P.done_out;
        f.done_need = (uint32_t)grid;
        // Norm weights gathered by mask (dense: the weights themselves).
        std::vector<uint16_t> nw((size_t)g.K);
        cudaError_t e = cudaMemcpy(nw.data(), g.norm_w, (size_t)g.K * 2, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return fail_cuda(e, "reading norm weights");
        const size_t nwc_off = ar.take_static((size_t)nsegx * g.w_pad * 2);
        for (int sx = 0; sx < nsegx; ++sx) {
          uint16_t* dst = reinterpret_cast<uint16_t*>(ar.init.data() + nwc_off) + (size_t)sx * g.w_pad;
          if (dense) {
            for (int j = 0; j < g.K; ++j) dst[j] = nw[j];
          } else {
            std::vector<uint8_t> idx;
            rc = read_mask(g, sx, &idx);
            if (rc) return rc;
            for (int j = 0; j < g.w; ++j) {
              const int col = (j / g.n) * g.m + (int)idx[j];
              if (col < g.K) dst[j] = nw[col];
            }
          }
        }
        f.nwc = flow_off<const __half>(nwc_off, false);
        rc = route_inputs(kOwnGemv, it->second.index);
        if (rc) return rc;
      } else {
        auto it = out_owner.find(g.x);
        if (it == out_owner.end())
          return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: input is not produced inside the step", i);
        if (it->second.kind == kOwnGemv) {
          nms::FlowGemv& P = fg[it->second.index];
          if (P.out_mode != -1 || P.sg.g.epilogue != nms::kEpiSwiGLU)
            return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: a plain input must come from a SwiGLU GEMV", i);
          P.out_mode = nms::kFlowOutAct;
          f.done_in = P.done_out;
          f.done_need = (uint32_t)grid;
        } else {
          f.done_in = fa[it->second.index].done_out;
          f.done_need = (uint32_t)fa[it->second.index].a.Hkv;  // one combining unit per KV head
        }
        rc = route_inputs(it->second.kind, it->second.index);
        if (rc) return rc;
      }
      if (g.epilogue == nms::kEpiArgmax) f.out_mode = nms::kFlowOutArgmax;
      size_t a0, a1, a2, a3, a4, a5, a6;
      const size_t need_sm = nms::flow_gemv_layout(g.K, g.w, g.w_pad, nsegx, max_vrows, norm,
                                                   f.in_mode == nms::kFlowInGather, &a0, &a1, &a2, &a3, &a4, &a5, &a6);
      if (need_sm > act) act = need_sm;
      if (((g.row_groups + grid - 1) / grid) * RG > NT && g.epilogue != nms::kEpiArgmax)
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: more than %d output rows per CTA", i, NT);
      nms::ProdDesc pd;
      memset(&pd, 0, sizeof(pd));
      for (int q = 0; q < g.nseg; ++q) {
        pd.w[q] = g.seg[q].w;
        pd.row_start[q] = g.seg[q].row_start;
      }
      pd.rows_total = g.rows_total;
      pd.row_groups = g.row_groups;
      pd.w_pad = g.w_pad;
      pd.nseg = (int16_t)g.nseg;
      pd.paired = paired ? 1 : 0;
      pd.lanes = (int8_t)sg.lanes;
      kinds.push_back(nms::kStageGemv);
      fg.push_back(f);
      descs.push_back(pd);
      natural_of_gemv.push_back(nullptr);
      if (g.epilogue != nms::kEpiArgmax) out_owner[g.out] = FlowOwner{kOwnGemv, gi};
    } else if (r.kind == LaunchRec::kAttention) {
      const int ai = (int)fa.size();
      nms::FlowAttn a;
      memset(&a, 0, sizeof(a));
      a.a = r.ap;
      const int units = a.a.Hkv * a.a.splits;
      if (a.a.splits > nms::kMaxSplits || units > grid)
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: %d attention units for %d CTAs", i, units, grid);
      if (pos_ptr == nullptr) pos_ptr = a.a.pos;
      if (a.a.pos != pos_ptr) return fail(NMS_ERR_VALUE, "record %d: attention stages must share one position", i);
      auto it = out_owner.find(a.a.qkv);
      const int qkv_rows = (a.a.Hq + 2 * a.a.Hkv) * nms::kAttnD;
      if (it == out_owner.end() || it->second.kind != kOwnGemv)
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: q/k/v are not produced inside the step", i);
      nms::FlowGemv& Q = fg[it->second.index];
      if (Q.out_mode != -1 || Q.sg.g.epilogue != nms::kEpiStore || Q.sg.g.rows_total != qkv_rows)
        return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: the q/k/v producer is not a plain %d-row GEMV", i, qkv_rows);
      Q.out_mode = nms::kFlowOutWords;
      a.done_in = Q.done_out;
      a.done_need = (uint32_t)grid;
      a.done_out = flow_off<unsigned>((size_t)(nstage_counter++) * 4, true);
      uint32_t* words = flow_off<uint32_t>(ar.take_dyn((size_t)qkv_rows * 4), true);
      natural_of_gemv[it->second.index] = words;
      a.qkv_in = words;
      const int G = a.a.Hq / a.a.Hkv;
      a.part = flow_off<unsigned long long>(ar.take_dyn((size_t)units * G * (nms::kAttnD + 2) * 8), true);
      kinds.push_back(nms::kStageAttn);
      fa.push_back(a);
      natural_of_attn.push_back(nullptr);
      out_owner[a.a.y] = FlowOwner{kOwnAttn, ai};
    } else {
      return fail(NMS_ERR_NOT_IMPLEMENTED, "record %d: only GEMV and attention launches run in a persistent step", i);
    }
  }
  for (size_t gi = 0; gi < fg.size(); ++gi) {
    if (fg[gi].out_mode == -1)
      return fail(NMS_ERR_NOT_IMPLEMENTED, "GEMV stage %zu: its output is not consumed inside the step", gi);
    fg[gi].out_words = natural_of_gemv[gi];
  }
  for (size_t ai = 0; ai < fa.size(); ++ai) fa[ai].y_words = natural_of_attn[ai];
  if (fg.empty() || kinds.back() != nms::kStageGemv || fg.back().out_mode != nms::kFlowOutArgmax)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "the step must end with the argmax head");

  // Shared memory: [rings][working set][stream descriptors][stage kinds].
  act = nms::align_up_sz(act, 128);
  const size_t tail_bytes = descs.size() * sizeof(nms::ProdDesc) + nms::align_up_sz(kinds.size() * 4, 16);
  const size_t ring_unit = (size_t)nms::kStepWarps * nms::kRingItemBytes;
  int depth = 0;
  for (int d : {nms::kStepDepthHi, nms::kStepDepthLo})
    if (depth == 0 && (size_t)d * ring_unit + act + tail_bytes <= dev->step_smem_max) depth = d;
  if (depth == 0)
    return fail(NMS_ERR_NOT_IMPLEMENTED, "flow step: a %zu-byte working set leaves no room for the weight rings", act);

  const size_t kind_off = ar.take_dyn(kinds.size() * 4);
  const size_t gemv_off = ar.take_dyn(fg.size() * sizeof(nms::FlowGemv));
  const size_t desc_off = ar.take_dyn(descs.size() * sizeof(nms::ProdDesc));
  const size_t attn_off = ar.take_dyn(std::max<size_t>(1, fa.size()) * sizeof(nms::FlowAttn));
  const size_t ctl_off = ar.take_dyn(256);  // exit counter at +0, spare word at +64, epoch at +128
  const size_t cnt_off = ar.take_dyn((size_t)std::max(1, nstage_counter) * 4);
  const size_t static_bytes = nms::align_up_sz(ar.static_end, 256);
  const size_t total = static_bytes + ar.end;

  nms_step* st = new (std::nothrow) nms_step();
  if (st == nullptr) return fail(NMS_ERR_CUDA, "out of host memory");
  cudaError_t e = cudaGetDevice(&st->device);
  if (e == cudaSuccess) e = cudaMalloc(&st->dev_mem, total);
  if (e == cudaSuccess) e = cudaMemset(st->dev_mem, 0, total);
  unsigned char* base = static_cast<unsigned char*>(st->dev_mem);
  auto dyn_addr = [&](size_t off) { return base + static_bytes + off; };
  auto patch = [&](auto*& ptr) {
    if (ptr == nullptr) return;
    const uintptr_t v = reinterpret_cast<uintptr_t>(ptr);
    const size_t off = (size_t)((v & ~kFlowDynBit) - 1);
    unsigned char* a = (v & kFlowDynBit) ? base + static_bytes + off : base + off;
    ptr = reinterpret_cast<std::remove_reference_t<decltype(ptr)>>(a);
  };
  // Completion counters were numbered, not placed: rebase them onto their block.
  auto patch_cnt = [&](auto*& ptr) {
    if (ptr == nullptr) return;
    const size_t idx = (size_t)(((reinterpret_cast<uintptr_t>(ptr) & ~kFlowDynBit) - 1) / 4);
    ptr = reinterpret_cast<std::remove_reference_t<decltype(ptr)>>(dyn_addr(cnt_off) + idx * 4);
  };
  for (nms::FlowGemv& f : fg) {
    patch_cnt(f.done_in);
    patch_cnt(f.done_out);
  }
  for (nms::FlowAttn& a : fa) {
    patch_cnt(a.done_in);
    patch_cnt(a.done_out);
  }
  for (nms::FlowGemv& f : fg) {
    for (int q = 0; q < nms::kMaxSegs; ++q) patch(f.xc_in[q]);
    patch(f.nwc);
    patch(f.ssq_in);
    patch(f.gather_resid);
    patch(f.out_words);
    patch(f.resid_old);
    patch(f.ssq_out);
    for (int q = 0; q < nms::kFlowMaxScat; ++q) {
      patch(f.scat_dst[q]);
      patch(f.scat_inv[q]);
    }
  }
  for (nms::FlowAttn& a : fa) {
    patch(a.qkv_in);
    patch(a.part);
    patch(a.y_words);
    patch(a.y_dst);
    patch(a.y_inv);
  }
  if (e == cudaSuccess && ar.static_end > 0) e = cudaMemcpy(base, ar.init.data(), ar.static_end, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dyn_addr(kind_off), kinds.data(), kinds.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(dyn_addr(gemv_off), fg.data(), fg.size() * sizeof(nms::FlowGemv), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(dyn_addr(desc_off), descs.data(), descs.size() * sizeof(nms::ProdDesc), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && !fa.empty())
    e = cudaMemcpy(dyn_addr(attn_off), fa.data(), fa.size() * sizeof(nms::FlowAttn), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (st->dev_mem) cudaFree(st->dev_mem);
    delete st;
    return fail_cuda(e, "flow step set-up");
  }
  st->flow = true;
  st->nstages = (int)kinds.size();
  st->grid = grid;
  st->depth = depth;
  st->smem = (size_t)depth * ring_unit + act + tail_bytes;
  nms::FlowParams& F = st->fparams;
  memset(&F, 0, sizeof(F));
  F.kind = reinterpret_cast<const int32_t*>(dyn_addr(kind_off));
  F.gemv = reinterpret_cast<const nms::FlowGemv*>(dyn_addr(gemv_off));
  F.desc = reinterpret_cast<const nms::ProdDesc*>(dyn_addr(desc_off));
  F.attn = reinterpret_cast<const nms::FlowAttn*>(dyn_addr(attn_off));
  F.nstages = st->nstages;
  F.ngemv = (int32_t)fg.size();
  F.nattn = (int32_t)fa.size();
  F.ring_bytes = (int32_t)((size_t)depth * ring_unit);
  F.act_bytes = (int32_t)act;
  F.exit_count = reinterpret_cast<unsigned*>(dyn_addr(ctl_off));
  F.counters = reinterpret_cast<unsigned*>(dyn_addr(cnt_off));
  F.ncounters = nstage_counter;
  F.spare = reinterpret_cast<unsigned*>(dyn_addr(ctl_off) + 64);
  F.epoch = reinterpret_cast<unsigned long long*>(dyn_addr(ctl_off) + 128);
  F.pos = pos_ptr;
  memset(&st->params, 0, sizeof(st->params));
  // nms_step_reset zeroes the exit counter and the spare word; the epoch
  // keeps counting (tags stay unique).
  st->params.bar_count = F.exit_count;
  st->params.attn_count = F.counters;
  st->bar_bytes = 4;
  st->cnt_bytes = (size_t)std::max(1, nstage_counter) * 4;
  st->gemv_of_stage.assign(kinds.size(), -1);
  *out = st;
  return NMS_OK;
}

int64_t nms_tp_area_bytes(int32_t nreduce, int32_t world, int32_t dim) {
  if (nreduce < 1 || world < 1 || dim < 1) return -1;
  return 256 + (int64_t)(nreduce + 1) * world * (dim < 2 ? 2 : dim) * 8;  // + the head's candidate point
}

int nms_ipc_alloc(int64_t bytes, void** ptr_out, void* handle_out) {
  if (bytes <= 0 || ptr_out == nullptr || handle_out == nullptr) return fail(NMS_ERR_VALUE, "bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail_cuda(e, "exchange area allocation");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return NMS_OK;
}

int nms_ipc_free(void* ptr) {
  if (ptr == nullptr) return NMS_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? NMS_OK : fail_cuda(e, "cudaFree");
}

int nms_ipc_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return fail(NMS_ERR_VALUE, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? NMS_OK : fail_cuda(e, "cudaIpcOpenMemHandle");
}

int nms_ipc_close(void* ptr) {
  if (ptr == nullptr) return NMS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? NMS_OK : fail_cuda(e, "cudaIpcCloseMemHandle");
}

int nms_step_set_tp(nms_step* step, const int32_t* reduce_stages, int32_t nreduce, const nms_tp_config* cfg) {
  if (step == nullptr || reduce_stages == nullptr || cfg == nullptr) return fail(NMS_ERR_VALUE, "null argument");
  if (cfg->world < 2 || cfg->world > NMS_MAX_TP || cfg->rank < 0 || cfg->rank >= cfg->world)
    return fail(NMS_ERR_VALUE, "world=%d rank=%d (2 <= world <= %d)", cfg->world, cfg->rank, NMS_MAX_TP);
  if (nreduce < 1 || cfg->dim < 2) return fail(NMS_ERR_VALUE, "nreduce=%d dim=%d", nreduce, cfg->dim);
  if (step->params.tp_world > 1) return fail(NMS_ERR_VALUE, "tensor parallelism is already set for this step");
  if (step->flow) return fail(NMS_ERR_NOT_IMPLEMENTED, "tensor parallelism runs on the barrier step (nms_step_create)");
  for (int r = 0; r < cfg->world; ++r)
    if (cfg->area[r] == nullptr || !aligned(cfg->area[r], 256)) return fail(NMS_ERR_VALUE, "area %d missing or unaligned", r);
  std::vector<nms::StepGemv> g = step->gemvs;
  for (nms::StepGemv& sg : g) sg.tp_send = sg.tp_recv = -1;
  int last = -1;
  for (int j = 0; j < nreduce; ++j) {
    const int s = reduce_stages[j];
    if (s <= last || s >= step->nstages) return fail(NMS_ERR_VALUE, "reduce stages must ascend inside the step");
    last = s;
    const int gi = step->gemv_of_stage[s];
    if (gi < 0) return fail(NMS_ERR_VALUE, "stage %d is not a GEMV", s);
    nms::StepGemv& snd = g[gi];
    if (snd.g.epilogue != nms::kEpiStore || snd.g.mode == nms::kModePaired || snd.g.rows_total != cfg->dim)
      return fail(NMS_ERR_VALUE, "stage %d: an exchange point must store %d rows", s, cfg->dim);
    snd.tp_send = j;
    // The next GEMV stage adds the reduced vector as its residual addend.
    for (int k = s + 1; k < step->nstages; ++k) {
      const int gk = step->gemv_of_stage[k];
      if (gk < 0) continue;
      nms::StepGemv& rcv = g[gk];
      if (rcv.g.prologue != nms::kProResidNorm || rcv.g.x2 != snd.g.out || rcv.g.K != cfg->dim)
        return fail(NMS_ERR_VALUE, "stage %d: the GEMV after exchange point %d must take it as residual addend", k, j);
      rcv.tp_recv = j;
      break;
    }
  }
  // A vocabulary-parallel argmax head as the last stage: the local winner
  // goes to a scratch word and the kernel's tail swaps candidates.
  const int last_g = step->gemv_of_stage[step->nstages - 1];
  const bool head = last_g >= 0 && g[last_g].g.epilogue == nms::kEpiArgmax;
  if (head) {
    nms::GemvParams& hp = g[last_g].g;
    step->params.tp_token_out = hp.token_out;
    step->params.tp_next_token = hp.next_token;
    step->params.tp_history = hp.token_history;
    step->params.tp_pos = hp.pos;
    step->params.tp_history_len = hp.history_len;
    step->params.tp_local_best = reinterpret_cast<int64_t*>(reinterpret_cast<unsigned char*>(step->params.bar_count) + 192);
    hp.token_out = step->params.tp_local_best;
    hp.next_token = nullptr;
    hp.token_history = nullptr;
    hp.pos = nullptr;
  }
  const size_t cbytes = 256;  // the step counter, then the values
  nms::StepParams& P = step->params;
  cudaError_t e = cudaSetDevice(step->device);
  if (e == cudaSuccess)
    e = cudaMemcpy(const_cast<nms::StepGemv*>(P.gemv), g.data(), g.size() * sizeof(nms::StepGemv),
                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail_cuda(e, "tensor-parallel stage table");
  P.tp_world = cfg->world;
  P.tp_rank = cfg->rank;
  P.tp_head = head ? 1 : 0;
  P.tp_vocab_offset = cfg->vocab_offset;
  P.tp_dim = cfg->dim;
  P.tp_nreduce = nreduce;
  for (int r = 0; r < nms::kMaxTp; ++r) {
    unsigned char* a = r < cfg->world ? static_cast<unsigned char*>(cfg->area[r]) : nullptr;
    // area: [steps completed] (padded to 256 bytes), then {fp32, tag} values
    P.tp_vals[r] = a ? reinterpret_cast<uint2*>(a + cbytes) : nullptr;
  }
  unsigned char* mine = static_cast<unsigned char*>(cfg->area[cfg->rank]);
  P.tp_epoch = reinterpret_cast<unsigned long long*>(mine);
  P.tp_my_vals = reinterpret_cast<const uint2*>(mine + cbytes);
  step->gemvs = g;
  return NMS_OK;
}

int nms_step_launch(const nms_step* step, void* stream) {
  if (step == nullptr) return fail(NMS_ERR_VALUE, "step is null");
  if (step->flow) {
    cudaError_t e = launch_ex2(step->depth == nms::kStepDepthHi ? nms::decode_flow_kernel<nms::kStepDepthHi>
                                                               : nms::decode_flow_kernel<nms::kStepDepthLo>,
                               dim3(step->grid), dim3(nms::kStepThreads), step->smem,
                               static_cast<cudaStream_t>(stream), false, dim3(1, 1, 1), true, step->fparams);
    if (e != cudaSuccess) return fail_cuda(e, "decode_flow_kernel launch");
    return NMS_OK;
  }
  cudaError_t e = launch_ex2(step->depth == nms::kStepDepthHi ? nms::decode_step_kernel<nms::kStepDepthHi>
                                                             : nms::decode_step_kernel<nms::kStepDepthLo>,
                             dim3(step->grid), dim3(nms::kStepThreads), step->smem, static_cast<cudaStream_t>(stream),
                             false, dim3(1, 1, 1), true, step->params);
  if (e != cudaSuccess) return fail_cuda(e, "decode_step_kernel launch");
  return NMS_OK;
}

int nms_step_reset(const nms_step* step, void* stream) {
  if (step == nullptr) return fail(NMS_ERR_VALUE, "step is null");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(step->params.bar_count, 0, step->bar_bytes, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(step->params.attn_count, 0, step->cnt_bytes, st);
  if (e != cudaSuccess) return fail_cuda(e, "persistent step counter reset");
  return NMS_OK;
}

int nms_step_set_trace(nms_step* step, void* buffer, int64_t capacity) {
  if (step == nullptr) return fail(NMS_ERR_VALUE, "step is null");
  if (buffer == nullptr) {
    step->params.trace = nullptr;
    step->params.trace_detail = nullptr;
    step->fparams.trace = nullptr;
    step->fparams.trace_detail = nullptr;
    return NMS_OK;
  }
  const int64_t need = 1 + (int64_t)step->nstages * (step->grid + 1);
  if (capacity < need) return fail(NMS_ERR_VALUE, "trace needs %lld entries, got %lld", (long long)need, (long long)capacity);
  if (!aligned(buffer, 8)) return fail(NMS_ERR_VALUE, "trace buffer must be 8-byte aligned");
  step->params.trace = static_cast<unsigned long long*>(buffer);
  const int64_t detail = (int64_t)step->nstages * step->grid * nms::kTraceMarks;
  step->params.trace_detail = capacity >= need + detail ? step->params.trace + need : nullptr;
  step->fparams.trace = step->params.trace;
  step->fparams.trace_detail = step->params.trace_detail;
  return NMS_OK;
}

int nms_step_info(const nms_step* step, int32_t* nstages, int32_t* grid) {
  if (step == nullptr || nstages == nullptr || grid == nullptr) return fail(NMS_ERR_VALUE, "null argument");
  *nstages = step->nstages;
  *grid = step->grid;
  return NMS_OK;
}

int nms_step_destroy(nms_step* step) {
  if (step == nullptr) return NMS_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(step->device);
  if (step->dev_mem) cudaFree(step->dev_mem);
  cudaSetDevice(cur);
  delete step;
  return NMS_OK;
}

int nms_gemm_workspace_bytes(int64_t T, int64_t w_pad, int64_t h, int64_t* bytes_out) {
  if (bytes_out == nullptr) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (T <= 0 || h <= 0 || w_pad <= 0 || w_pad % 64 != 0)
    return fail(NMS_ERR_VALUE, "T, h must be positive and w_pad a positive multiple of 64");
  const DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  GemmPlan g;
  rc = gemm_plan(T, w_pad, h, dev->num_sms, dev->gemm_smem_max, &g);
  if (rc) return rc;
  *bytes_out = g.total;
  return NMS_OK;
}

int nms_gemm_packed_f16(const void* x, int32_t x_dtype, const void* packed, const void* mat_index, void* out,
                        int64_t T, int64_t K, int64_t w, int64_t w_pad, int64_t h, int32_t block_width,
                        int32_t vec_width, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!x || !packed || !mat_index || !out || !workspace) return fail(NMS_ERR_VALUE, "null pointer argument");
  if (x_dtype != NMS_DTYPE_F16 && x_dtype != NMS_DTYPE_BF16 && x_dtype != NMS_DTYPE_F32)
    return fail(NMS_ERR_TYPE, "x_dtype=%d is not NMS_DTYPE_F16/BF16/F32", x_dtype);
  int rc = gemm_check_shape(T, K, w, w_pad, h, block_width, vec_width);
  if (rc) return rc;
  if (!aligned(packed, 16)) return fail(NMS_ERR_VALUE, "packed must be 16-byte aligned");
  if (!aligned(workspace, 256)) return fail(NMS_ERR_VALUE, "workspace must be 256-byte aligned");
  const int esize = x_dtype == NMS_DTYPE_F32 ? 4 : 2;
  if (!aligned(x, esize)) return fail(NMS_ERR_VALUE, "x is not aligned to its element size");
  if (!aligned(out, 2)) return fail(NMS_ERR_VALUE, "out must be 2-byte aligned");
  const DeviceInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  GemmPlan g;
  rc = gemm_plan(T, w_pad, h, dev->num_sms, dev->gemm_smem_max, &g);
  if (rc) return rc;
  if (workspace_bytes < g.total)
    return fail(NMS_ERR_VALUE, "workspace of %lld bytes < %lld required (nms_gemm_workspace_bytes)",
                (long long)workspace_bytes, (long long)g.total);
  __half* xc = static_cast<__half*>(workspace);

  CUtensorMap tm_a, tm_b;
  rc = encode_k_major(&tm_a, packed, h, w_pad, nms::kGemmBM);
  if (rc) return rc;
  rc = encode_k_major(&tm_b, xc, T, w_pad, g.bn);
  if (rc) return rc;

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned gblocks = (unsigned)((T * (w_pad / 8) + 255) / 256);
  const uint8_t* idx = static_cast<const uint8_t*>(mat_index);
  if (x_dtype == NMS_DTYPE_F16)
    nms::gather_xc_kernel<__half><<<gblocks, 256, 0, st>>>(static_cast<const __half*>(x), idx, xc, (int32_t)T,
                                                           (int32_t)K, (int32_t)w, (int32_t)w_pad, block_width,
                                                           vec_width);
  else if (x_dtype == NMS_DTYPE_BF16)
    nms::gather_xc_kernel<__nv_bfloat16><<<gblocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), idx, xc,
                                                                  (int32_t)T, (int32_t)K, (int32_t)w, (int32_t)w_pad,
                                                                  block_width, vec_width);
  else
    nms::gather_xc_kernel<float><<<gblocks, 256, 0, st>>>(static_cast<const float*>(x), idx, xc, (int32_t)T,
                                                          (int32_t)K, (int32_t)w, (int32_t)w_pad, block_width,
                                                          vec_width);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "gather_xc_kernel launch");

  nms::GemmParams p;
  p.out = static_cast<__half*>(out);
  p.T = (int32_t)T;
  p.h = (int32_t)h;
  p.bn = g.bn;
  p.atoms = g.atoms;
  p.kblocks = g.kblocks;
  p.splits = g.splits;
  p.stages = g.stages;
  p.idesc = nms::umma_idesc_f16_f32(nms::kGemmBM, g.bn);
  p.tmem_cols = 32;
  while ((int32_t)p.tmem_cols < g.bn) p.tmem_cols <<= 1;
  p.vec_out = (h % 8 == 0 && aligned(out, 16)) ? 1 : 0;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)g.m_tiles, (unsigned)g.n_tiles, (unsigned)g.splits);
  cfg.blockDim = dim3(nms::kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)g.splits;  // the k-splits of one tile form a cluster
  // Programmatic dependent of the gather: the prologue and the first weight
  // tiles overlap it; xc is read only after griddepcontrol.wait.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, nms::gemm_nm_kernel, tm_a, tm_b, p);
  if (e != cudaSuccess) return fail_cuda(e, "gemm_nm_kernel launch");
  return NMS_OK;
}

int nms_plan_launch(const nms_plan* plan, int32_t begin, int32_t end, void* stream) {
  if (plan == nullptr) return fail(NMS_ERR_VALUE, "plan is null");
  const int32_t n = (int32_t)plan->recs.size();
  if (begin < 0 || end > n || begin > end) return fail(NMS_ERR_VALUE, "range [%d, %d) outside plan of %d", begin, end, n);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int32_t i = begin; i < end; ++i) {
    int rc = launch_rec(plan->recs[i], st);
    if (rc) return rc;
  }
  return NMS_OK;
}

}  // extern "C"
