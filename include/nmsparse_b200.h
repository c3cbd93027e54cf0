/*
 * nmsparse_b200.h -- C ABI of libnmsparse_b200.so, the B200 (sm_100a) N:M
 * sparse GEMV decode path.
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise; all tensors
 *     are dense and contiguous; fp16 means IEEE binary16.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Calls enqueue work and return without synchronizing.
 *   - Every function returns an nms_status (0 = success).  On failure nothing
 *     is launched and nms_last_error() returns a message for the calling
 *     thread.  The Python layer maps NMS_ERR_VALUE -> ValueError,
 *     NMS_ERR_TYPE -> TypeError, NMS_ERR_NOT_IMPLEMENTED ->
 *     NotImplementedError and the others -> RuntimeError, the exception types
 *     the reference raises for the same conditions (triton_spmv.py:245-283).
 *
 * Layouts (w = K*N/M compressed width, G = K/M groups, h = output rows)
 *   mat_data  fp16 [w, h]   reference layout, element (j, r) at j*h + r
 *                            (triton_spmv.py:10-13, src/spmv/nmsparse_linear.py:22-24)
 *   mat_index u8   [G, N]   sorted in-group offsets shared by all rows
 *                            (src/spmv/nmsparse_linear.py:22-26)
 *   packed    fp16 [h, w_pad] row-major transpose of mat_data, rows zero
 *                            padded to w_pad = nms_packed_row_stride(w)
 */
#ifndef NMSPARSE_B200_H_
#define NMSPARSE_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NMS_ABI_VERSION 2

enum nms_status {
  NMS_OK = 0,
  NMS_ERR_VALUE = -1,           /* bad shape, size, pointer or alignment   */
  NMS_ERR_TYPE = -2,            /* unsupported dtype                       */
  NMS_ERR_NOT_IMPLEMENTED = -3, /* valid request outside what is built     */
  NMS_ERR_CUDA = -4,            /* CUDA runtime error                      */
  NMS_ERR_DEVICE = -5           /* a kernel reported an error (see below)  */
};

int nms_abi_version(void);
/* SHA-256 (hex) of the sources the library was built from (csrc/ and this
 * header), so a caller can refuse a library that is older than its sources.
 * No reference counterpart (the reference JIT-compiles its Triton kernel). */
const char* nms_source_hash(void);
const char* nms_last_error(void);
const char* nms_status_name(int status);
/* Number of SMs of the current device (also checks it is an sm_100 part). */
int nms_num_sms(int* out);
/* Reads the device error word that kernels set instead of faulting or
 * hanging (1 = bulk-copy wait timed out, 2 = attention position outside the
 * KV cache, 3 = persistent-step grid barrier timed out, 4 = persistent-step
 * weight-ring slot never refilled, 5 = persistent-step weight-ring chunk does
 * not fit its stage, 6 = prefill GEMM copy or tensor-core wait timed out; the
 * kernel skipped its work).  Synchronizes the current
 * device.  With clear != 0 the word is reset to 0. */
int nms_device_error(int* code_out, int clear);
/* Host-side abort request: sets the device error word to `code` (> 0).
 * Kernels of this library that are inside a bounded wait (persistent-step
 * grid barriers and tensor-parallel exchanges) give up at once and leave;
 * a launch that starts while the word is set abandons its first barrier.
 * The word stays set until nms_device_error(.., clear=1).  No reference
 * counterpart: it lets a watchdog end a stuck step without a GPU fault. */
int nms_device_error_set(int code);

/* ---------------------------------------------------------------------------
 * Shared-mask N:M GEMV on the reference layout.
 * Replaces nmsparse_spmv_forward_triton_ptx (triton_spmv.py:229-318) and the
 * triton_ptx branch of the nmsparse::gemv op (src/spmv/nmsparse_op.py:82-96):
 *   out[r] = sum_g sum_i mat_data[g*N + i, r] * vec[g*M + mat_index[g, i]]
 * fp16 in, fp32 accumulation, fp16 out.  No zero-initialised fp32 scratch
 * and no separate cast kernel: out is written once.
 *   vec [K] fp16, mat_data [w, h] fp16 (32-byte aligned), mat_index [w/N, N],
 *   out [h] fp16.  Requires h % 128 == 0, w % N == 0, K == (w/N)*M, M <= 256.
 * ------------------------------------------------------------------------- */
int nms_gemv_f16(const void* vec, const void* mat_data, const void* mat_index, void* out, int64_t K,
                 int64_t w, int64_t h, int32_t block_width, int32_t vec_width, void* stream);

/* Per-row N:M on the reference layout: the non-shared index layout of
 * src/spmv/nmsparse_linear.py:27-29 (mat_index u8 [w, h], element (j, r) at
 * j*h + r, each row with its own in-group offsets; the reference ships no
 * kernel for it, src/spmv/nmsparse_op.py:33-44,98-116):
 *   out[r] = sum_j mat_data[j, r] * vec[(j/N)*M + mat_index[j, r]]
 * Same shape rules as nms_gemv_f16; mat_index 16-byte aligned; K <= ~110k. */
int nms_gemv_rowwise_f16(const void* vec, const void* mat_data, const void* mat_index, void* out, int64_t K,
                         int64_t w, int64_t h, int32_t block_width, int32_t vec_width, void* stream);

/* ---------------------------------------------------------------------------
 * Packed layout (the re-laid-out packer; no reference counterpart: the
 * reference streams mat_data[w, h] directly, triton_spmv.py:100-106).
 * nms_pack_f16 / nms_unpack_f16 convert between mat_data[w, h] and
 * packed[h, w_pad]; the round trip is bit-exact.
 * ------------------------------------------------------------------------- */
int64_t nms_packed_row_stride(int64_t w);
int nms_pack_f16(const void* mat_data, void* packed, int64_t w, int64_t h, int64_t w_pad, void* stream);
int nms_unpack_f16(const void* packed, void* mat_data, int64_t w, int64_t h, int64_t w_pad, void* stream);

/* Same GEMV as nms_gemv_f16 on the packed layout (any h >= 1).  Used by
 * NmSparseLinear.forward for single-token input
 * (src/spmv/nmsparse_linear.py:62-66). */
int nms_gemv_packed_f16(const void* vec, const void* packed, const void* mat_index, void* out, int64_t K,
                        int64_t w, int64_t w_pad, int64_t h, int32_t block_width, int32_t vec_width,
                        void* stream);

/* ---------------------------------------------------------------------------
 * Batch > 1 (prefill) sparse GEMM on the packed layout.  The reference sends
 * every multi-token input to a dense F.linear with the unpruned weight
 * (src/spmv/nmsparse_linear.py:55-68) and its op refuses rows != 1
 * (src/spmv/nmsparse_op.py:84-87); this computes the sparse layer itself:
 *   out[t, r] = sum_j packed[r, j] * x[t, (j/N)*M + mat_index[j/N, j%N]]
 * for T tokens: x [T, K] (x_dtype: fp16, bf16 or fp32, converted to fp16 as
 * the reference op converts its input), packed [h, w_pad] fp16 (16-byte
 * aligned), out [T, h] fp16, fp32 accumulation on the tensor cores.
 * workspace: caller-owned device memory of nms_gemm_workspace_bytes(T, w_pad,
 * h) bytes (256-byte aligned; no initial contents needed).  Launches two
 * kernels on `stream` (gather + GEMM) and is CUDA-graph capturable; launches
 * that share a workspace must be ordered on one stream.  The result does not
 * depend on launch timing (split-K partials are summed in a fixed order).
 * ------------------------------------------------------------------------- */
#define NMS_DTYPE_F16 0
#define NMS_DTYPE_BF16 1
#define NMS_DTYPE_F32 2
int nms_gemm_workspace_bytes(int64_t T, int64_t w_pad, int64_t h, int64_t* bytes_out);
int nms_gemm_packed_f16(const void* x, int32_t x_dtype, const void* packed, const void* mat_index, void* out,
                        int64_t T, int64_t K, int64_t w, int64_t w_pad, int64_t h, int32_t block_width,
                        int32_t vec_width, void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Fused decode launches (packed layout).  One launch covers several linears
 * that read the same input vector:
 *   NMS_EPI_STORE   segments' outputs concatenated: q/k/v
 *                   (model.py:196-198,219 fused wqkv; HF q_proj/k_proj/v_proj)
 *   NMS_EPI_SWIGLU  two segments (gate, up) with equal rows:
 *                   out = silu(gate(x)) * up(x)        (model.py:255-256)
 *   NMS_EPI_ARGMAX  dense (NMS_FLAG_DENSE) output head: logits and greedy
 *                   token = argmax(logits), lowest index on ties
 *                   (model.py:168-169, generate.py:46-63 with greedy choice)
 * Prologue NMS_PRO_RESID_RMSNORM computes xin = fp16(x + x2) (x2 may be
 * NULL), writes xin to resid_out (if not NULL) and feeds
 * rmsnorm(xin) * norm_weight to the GEMV (model.py:185-188, 259-270).
 * Each segment may carry its own mat_index (masks differ per linear,
 * src/spmv/nmsparse_linear.py:118).
 * ------------------------------------------------------------------------- */
#define NMS_MAX_SEGMENTS 4
#define NMS_EPI_STORE 0
#define NMS_EPI_SWIGLU 1
#define NMS_EPI_ARGMAX 2
#define NMS_PRO_PLAIN 0
#define NMS_PRO_RESID_RMSNORM 1
#define NMS_FLAG_PDL 1   /* launch with programmatic dependent launch */
#define NMS_FLAG_DENSE 2 /* dense rows: w == K, mat_index must be NULL */
/* Launches without prefetch_bytes run the shared-memory ring kernel: one or
 * two 384-thread CTAs per SM, each at most half an SM; every warp streams its
 * weights through its own ring of 1 KB cp.async slots, filled before the
 * dependency wait, and the CTA lets its dependents launch at once, so with
 * NMS_FLAG_PDL a launch's start-up overlaps the previous launch's stream.
 * NMS_FLAG_REGISTER_RING selects the register-ring kernel instead (also used
 * with the L2 look-ahead, and when the rings do not fit).  Either kernel reads
 * weights, mask offsets and RMSNorm weights before its dependency wait: they
 * must not be written by the kernel it depends on. */
#define NMS_FLAG_REGISTER_RING 4

typedef struct nms_segment {
  const void* packed;    /* [rows, w_pad] fp16, 32-byte aligned */
  const void* mat_index; /* [w/N, N] u8, or NULL for dense      */
  int64_t rows;
} nms_segment;

typedef struct nms_gemv_fused_args {
  nms_segment seg[NMS_MAX_SEGMENTS];
  int32_t nseg;
  int32_t epilogue; /* NMS_EPI_* */
  int32_t prologue; /* NMS_PRO_* */
  int32_t flags;    /* NMS_FLAG_* */
  int64_t K, w, w_pad;
  int32_t block_width, vec_width; /* N, M (ignored when dense) */
  const void* x;           /* [K] fp16 */
  const void* x2;          /* [K] fp16 or NULL (prologue addend) */
  const void* norm_weight; /* [K] fp16 (RMSNorm prologue) */
  float eps;
  void* resid_out; /* [K] fp16 or NULL */
  void* out;       /* [sum rows] fp16 (STORE/ARGMAX) or [rows] (SWIGLU) */
  /* argmax epilogue scratch: amax_capacity partials, a counter that must be
   * zero before the first launch (the kernel resets it), the token output */
  float* amax_val;
  int32_t* amax_idx;
  uint32_t* amax_counter;
  int64_t* token_out;
  int32_t amax_capacity;
  int32_t grid;           /* CTAs (0 = two per SM) */
  int32_t prefetch_bytes; /* per-warp L2 look-ahead beyond the register ring (0 = off) */
  /* argmax generation hooks (each may be NULL): also write the token to
   * next_token; if pos is set, write token_history[*pos] = token (when
   * *pos < history_len) and then increment *pos.  Lets a captured decode
   * step feed itself (generate.py:93-119 decode_n_tokens loop). */
  int64_t* next_token;
  int64_t* token_history;
  int64_t* pos;
  int64_t history_len;
  /* Cross-launch L2 prefetch (optional): the weights of the launch that
   * follows this one, as up to two byte ranges; every CTA prefetches the
   * first next_prefetch_head bytes of its equal share of each range before
   * its dependency wait, so the next launch starts on L2 hits. */
  const void* next_prefetch[2];
  int64_t next_prefetch_bytes[2];
  int64_t next_prefetch_head;
  /* Token-indexed input (optional): x is a [x_rows, K] table and the GEMV
   * input is its row *x_token, read on the device -- the token embedding
   * (model.py:164) folded into the first GEMV of a decode step. */
  const int64_t* x_token;
  int64_t x_rows;
  /* Temperature sampling (NMS_EPI_ARGMAX only; temperature 0 = greedy): the
   * token is argmax(logit / temperature + g), g Gumbel(0, 1) noise from
   * Philox4x32-10 keyed by sample_seed and counted by (vocabulary row +
   * sample_row_offset, *sample_pos) -- a sample of softmax(logit /
   * temperature), the reference's sample() without top_k
   * (generate.py:46-63: argmax(probs / q), q ~ Exp(1)).  sample_pos may be
   * NULL (position 0). */
  float temperature;
  uint64_t sample_seed;
  const int64_t* sample_pos;
  int64_t sample_row_offset;
} nms_gemv_fused_args;

int nms_gemv_fused_f16(const nms_gemv_fused_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * Single-token attention with KV-cache append (batch 1, head_dim 128).
 * Replaces Attention.forward after the qkv projection (model.py:219-242:
 * split, RoPE, KVCache.update, flex_attention/SDPA with GQA) and the HF
 * Qwen3 attention with q_norm/k_norm (bench_qwen_3_32b_fp16_fixed_ptx.py:
 * 331-355 via transformers).
 * ------------------------------------------------------------------------- */
#define NMS_ROPE_INTERLEAVED 0 /* gpt-fast pairs (2i, 2i+1), model.py:310-322 */
#define NMS_ROPE_HALF 1        /* HF rotate_half pairs (i, i + D/2)          */

typedef struct nms_attention_args {
  const void* qkv;     /* [Hq*D + 2*Hkv*D] fp16: q | k | v of the new token */
  void* k_cache;       /* [Hkv, S_max, D] fp16 */
  void* v_cache;       /* [Hkv, S_max, D] fp16 */
  const void* rope;    /* [S_max, D/2, 2] fp16 (cos, sin) */
  const void* q_norm;  /* [D] fp16 or NULL */
  const void* k_norm;  /* [D] fp16 or NULL */
  const int64_t* pos;  /* device scalar: position of the new token, < S_max */
  void* y;             /* [Hq*D] fp16 */
  int32_t Hq, Hkv, D, S_max;
  int32_t rope_style;
  int32_t splits; /* CTAs per KV head, 1..16 (0 = automatic) */
  float norm_eps;
  float scale; /* usually 1/sqrt(D) */
  int32_t flags; /* NMS_FLAG_PDL */
  const void* next_prefetch[2]; /* as in nms_gemv_fused_args */
  int64_t next_prefetch_bytes[2];
  int64_t next_prefetch_head;
} nms_attention_args;

int nms_attention_decode_f16(const nms_attention_args* args, void* stream);

/* x = table[token] (token read on the device).  Replaces tok_embeddings
 * (model.py:164). */
int nms_embedding_f16(const void* table, const int64_t* token, void* x, int64_t K, int64_t vocab, int32_t flags,
                      void* stream);

/* ---------------------------------------------------------------------------
 * Output head + greedy token without any allocation (no counterpart in the
 * reference, which allocates its scratch per call, triton_spmv.py:285).
 * Same computation as nms_gemv_fused_f16 with NMS_FLAG_DENSE and
 * NMS_EPI_ARGMAX: logits = head_weight [vocab, K] x rmsnorm(x + x2) (the
 * norm prologue runs when norm_weight is not NULL; x2 may be NULL), and
 * *token_out = argmax(logits), lowest index on ties.  For callers that cannot
 * allocate device memory per call -- a serving runtime that has reserved the
 * whole GPU for its own pools, or a bare C FFI caller without a caching
 * allocator, where a cudaMalloc/cudaFree pair per token would synchronize the
 * device and cost more than the head itself.  Its argmax scratch is a static
 * 8.5 KB device array inside the library (partials of at most 1024 CTAs;
 * larger launches return NMS_ERR_VALUE).  The first call on each device looks
 * up that array's device address and should come before any stream capture.
 * Calls share the array: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialized by the caller.
 * ------------------------------------------------------------------------- */
int nms_gemv_argmax_noalloc_f16(const void* x, const void* x2, const void* norm_weight, float eps,
                                const void* head_weight, int64_t vocab, int64_t K, void* logits, int64_t* token_out,
                                void* stream);

/* ---------------------------------------------------------------------------
 * Launch plans: a native executor for one decode step.  Launches are
 * validated and frozen when added; nms_plan_launch replays a range of them
 * on a stream with no per-launch validation, so a decode step costs one
 * call from the host (or one CUDA-graph replay of that call).  Replaces the
 * torch.compile + CUDAGraph capture of decode_one_token
 * (benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:155-170).
 * ------------------------------------------------------------------------- */
typedef struct nms_plan nms_plan;

int nms_plan_create(nms_plan** out);
int nms_plan_destroy(nms_plan* plan);
int nms_plan_add_gemv(nms_plan* plan, const nms_gemv_fused_args* args);
int nms_plan_add_attention(nms_plan* plan, const nms_attention_args* args);
int nms_plan_add_embedding(nms_plan* plan, const void* table, const int64_t* token, void* x, int64_t K,
                           int64_t vocab, int32_t flags);
int nms_plan_size(const nms_plan* plan, int32_t* out);
/* Launch records [begin, end) on `stream`. */
int nms_plan_launch(const nms_plan* plan, int32_t begin, int32_t end, void* stream);

/* ---------------------------------------------------------------------------
 * Persistent decode step: the GEMV and attention records listed in
 * `records` (plan indices, in execution order) run as stages of ONE
 * cooperative kernel (one 640-thread CTA per SM) separated by in-kernel grid
 * barriers; every warp streams its weights through a shared-memory ring whose
 * copies run ahead across stage boundaries.  Replaces the per-kernel decode
 * step of the plan (and, like it, the reference's compiled + graph-captured
 * decode_one_token).
 * Records other than GEMV and attention (embedding, pack) return
 * NMS_ERR_NOT_IMPLEMENTED, and the plan path is used.  nms_step_create
 * allocates the stage table and barrier/attention scratch once (device
 * memory, freed by nms_step_destroy); launches allocate nothing.  Barrier
 * waits are bounded (device error 3 on timeout) and end early once the
 * device error word is set; every CTA then still leaves through the exit
 * path that zeroes the barrier words (the step's outputs are void).
 * ------------------------------------------------------------------------- */
typedef struct nms_step nms_step;

int nms_step_create(const nms_plan* plan, const int32_t* records, int32_t nrecords, nms_step** out);
/* The same step as a dataflow kernel without grid barriers: each stage's
 * output travels as tagged words ({fp16 value, tag} in 32 bits; per-CTA
 * fp32 partials as {value, tag} in 64 bits) that are their own arrival
 * signal; the o- and down-projection epilogues own their rows of the
 * residual stream and scatter them straight into the next stage's N:M
 * compressed input (inverse tables built here from mat_index); the RMSNorm
 * statistic arrives as per-CTA partials added in CTA order.  The routing is
 * derived from the records by pointer identity (the x, x2, resid_out and
 * out vectors of the decode step, as DecodeEngine builds it); a plan it
 * cannot route returns NMS_ERR_NOT_IMPLEMENTED and nms_step_create applies.
 * Not combinable with nms_step_set_tp.  Waits are bounded (device error 3)
 * and end once the device error word is set.  No reference counterpart
 * (replaces the same compiled + graph-captured decode_one_token). */
int nms_step_create_flow(const nms_plan* plan, const int32_t* records, int32_t nrecords, nms_step** out);
int nms_step_launch(const nms_step* step, void* stream);
int nms_step_destroy(nms_step* step);
/* Zero the step's barrier and attention arrival counters on `stream`.  Every
 * CTA leaves through the same exit path, which resets them, even after an
 * abandoned wait; a step that stopped inside an attention stage can still
 * leave a head counter behind, so after a nonzero nms_device_error call this
 * before the next launch (DecodeEngine.check_device does). */
int nms_step_reset(const nms_step* step, void* stream);
/* Stage count and CTAs of a persistent step. */
int nms_step_info(const nms_step* step, int32_t* nstages, int32_t* grid);
/* Optional timeline of later launches (NULL disables), in %globaltimer ns:
 * buf[0] = kernel start; buf[1 + s*(grid+1) + c] = when CTA c finished the
 * work of stage s; buf[1 + s*(grid+1) + grid] = when CTA 0 left the barrier
 * after stage s.  Needs 1 + nstages*(grid+1) uint64 entries (device memory).
 * With nstages*grid*8 more entries, a per-CTA detail (SM clock cycles of
 * that CTA's clock64, for phase lengths within a stage) follows at
 * buf[1 + nstages*(grid+1) + (s*grid + c)*8 + k]: k = 0 stage entry; GEMV:
 * 1 input vector staged, 2 norm statistic done, 3 staged mask offsets / norm
 * weights ready, 4 gathered vector built; attention: 4 first unit's q/k/v
 * prepared; then 5 main work done (GEMV: weight items consumed; attention:
 * partial state published), 6 stage finished; 7 unused. */
int nms_step_set_trace(nms_step* step, void* buffer, int64_t capacity);

/* ---------------------------------------------------------------------------
 * Tensor-parallel persistent step (no reference counterpart: the reference
 * decodes on one GPU; replaces the NCCL all-reduce after o_proj / down_proj
 * that a gpt-fast tp.py would add).  One process per GPU.  Each rank
 * allocates an exchange area with nms_ipc_alloc, the ranks swap the 64-byte
 * handles (e.g. torch.distributed all_gather_object) and open each other's
 * areas with nms_ipc_open.  nms_step_set_tp then turns the GEMV stages listed
 * in `reduce_stages` (stage indices of the step, ascending: the row-parallel
 * o- and down-projections) into exchange points: every CTA writes its fp32
 * partial rows into every rank's area over NVLink, each as one 8-byte
 * {value, tag} store whose tag names the step and point, so the data are
 * their own arrival signal; the next GEMV stage adds the ranks' partials
 * (rank order, identical on every rank) in place of its residual addend;
 * after a final exchange point the reduced vector is also written to that
 * stage's output.  If the step ends with a vocabulary-parallel argmax head
 * (NMS_EPI_ARGMAX), the ranks swap their best (logit, global index) the same
 * way and every rank writes the global greedy token (largest logit, lowest
 * index on ties) and runs the head's generation hooks.  Waits are bounded
 * (device error 3).  Area layout: step counter (8 bytes, padded to 256) +
 * (nreduce + 1) x world x dim {fp32, u32 tag}.
 * ------------------------------------------------------------------------- */
#define NMS_MAX_TP 8
typedef struct nms_tp_config {
  int32_t world, rank;
  int32_t dim;                   /* length of every reduced vector */
  int32_t vocab_offset;          /* first vocabulary row of this rank's head shard */
  void* area[NMS_MAX_TP];        /* every rank's exchange area, as mapped in this process */
} nms_tp_config;

/* Bytes of an exchange area for `nreduce` points of `dim` values over `world` ranks. */
int64_t nms_tp_area_bytes(int32_t nreduce, int32_t world, int32_t dim);
/* cudaMalloc'd, zeroed device memory and its IPC handle (64 bytes). */
int nms_ipc_alloc(int64_t bytes, void** ptr_out, void* handle_out);
int nms_ipc_free(void* ptr);
/* Map another process's allocation (its 64-byte handle) into this one. */
int nms_ipc_open(const void* handle, void** ptr_out);
int nms_ipc_close(void* ptr);
int nms_step_set_tp(nms_step* step, const int32_t* reduce_stages, int32_t nreduce, const nms_tp_config* cfg);

#ifdef __cplusplus
}
#endif

#endif /* NMSPARSE_B200_H_ */
