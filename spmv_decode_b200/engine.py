"""Fused batch-1 decode step on sm_100a: the engine behind decode_one_token.

A ``DecodeEngine`` takes a ``Transformer`` whose linears are
``NmSparseLinear`` (after ``swap_to_nmsparse``) or dense ``nn.Linear``, and
freezes one decode step into a native launch plan (libnmsparse_b200
``nms_plan_*``), replayed by a CUDA graph.  Per layer:

  1. q/k/v GEMV (one launch; fused wqkv or three masks) with the residual
     add + RMSNorm prologue                  model.py:185-186, 215-219
  2. attention: q/k RMSNorm, RoPE, KV append, split-KV softmax(QK^T)V
                                             model.py:221-242
  3. o-projection GEMV                       model.py:244
  4. gate/up GEMV with the residual + RMSNorm prologue and SwiGLU epilogue
                                             model.py:187, 255-256
  5. down-projection GEMV                    model.py:256
and finally the residual + final RMSNorm + dense output head with a greedy
argmax epilogue (model.py:168-169; generate.py:46-63 with greedy choice).
The token embedding gather starts the step (model.py:164).  Every kernel is
launched with programmatic dependent launch, so a kernel's weight stream
starts while its predecessor finishes.

Under tensor parallelism (``tp.TensorParallel``) each rank owns a column
shard of q/k/v and gate/up and a row shard of o/down; the plan is cut after
the o and down projections where an all-reduce of the partial sums runs.
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .model import Transformer, precompute_rope_table
from .nmsparse_linear import NmSparseLinear, sparse_prefill

ARGMAX_CAPACITY = 2048
# Persistent kernels tried before the barrier kernel in modes "auto" and
# "persistent" (the dataflow kernel, when enabled).
FLOW_DEFAULT: List[str] = []
# Mode "auto": below this many GEMV weight bytes per layer the plan executor
# (one launch per kernel, programmatic dependent launch) is faster than the
# persistent step, whose fixed cost per stage boundary weighs more the
# smaller the layer.  Measured on one B200 (ms/token, persistent / plan; CUDA
# graph replay, then with host I/O every step): Qwen3-0.6B 32:64 (16 MB per
# layer) 1.136 / 0.830, 1.166 / 0.885; Llama-3.1-8B 32:64 (218 MB)
# 2.181 / 2.106, 2.214 / 2.176; Qwen3-32B 16:32 (488 MB) 7.187 / 7.716,
# 7.261 / 7.835.
AUTO_PLAN_BELOW_LAYER_BYTES = 320 << 20


def auto_executor(layer_gemv_bytes: float) -> str:
    """The executor mode "auto" picks for a model with this many GEMV
    weight bytes per decoder layer: "plan" or "persistent"."""
    return "plan" if layer_gemv_bytes < AUTO_PLAN_BELOW_LAYER_BYTES else "persistent"

# Device error codes (include/nmsparse_b200.h, nms_device_error).
DEVICE_ERRORS = {
    1: "bulk-copy wait timed out",
    2: "token position outside the KV cache",
    3: "grid barrier or tensor-parallel exchange wait timed out",
    4: "weight-ring slot never refilled",
    5: "weight-ring chunk does not fit its stage",
    6: "prefill GEMM copy or tensor-core wait timed out",
}


def _linear_segment(lin) -> dict:
    """Segment description (packed weights, mask, rows, shape) of a linear."""
    if isinstance(lin, NmSparseLinear):
        if lin.layout != "shared":
            raise NotImplementedError(
                "the decode engine fuses shared-mask layers; per-row (layout='rowwise') layers decode "
                "through nmsparse::gemv in the model's own forward")
        return dict(packed=lin.mat_data, idx=lin.mat_index, rows=lin.h, K=lin.in_features, w=lin.w,
                    w_pad=lin.w_pad, n=lin.block_width, m=lin.vec_width, dense=False)
    if isinstance(lin, nn.Linear) or hasattr(lin, "weight"):
        wt = lin.weight
        if wt.dtype != torch.float16 or not wt.is_contiguous():
            raise TypeError("dense linears must hold contiguous float16 weights")
        rows, K = wt.shape
        return dict(packed=wt, idx=None, rows=rows, K=K, w=K, w_pad=K, n=1, m=1, dense=True)
    raise TypeError(f"unsupported linear {type(lin).__name__}")


class DecodeEngine:
    """Batch-1 decode state + native plan for one model on one device."""

    def __init__(self, model: Transformer, max_seq_length: int, *, pdl: bool = True, prefetch_bytes: int = 0,
                 next_prefetch_bytes: int = 0, attn_splits: int = 0, history_len: int = 0, mode: str = "auto",
                 allreduce: Optional[Callable[[torch.Tensor], None]] = None, tp_rank: int = 0, tp_size: int = 1,
                 local_heads: Optional[tuple] = None, head_hook: Optional[Callable[[bool], None]] = None,
                 temperature: float = 0.0, sample_seed: int = 0, vocab_offset: int = 0):
        c = model.config
        self.config = c
        self.model = model
        dev = model.tok_embeddings.weight.device
        if dev.type != "cuda":
            raise ValueError("DecodeEngine needs the model on a CUDA device")
        self.device = dev
        self.pdl = pdl
        self.prefetch_bytes = int(prefetch_bytes)  # per-warp L2 look-ahead inside a GEMV
        self.next_prefetch_bytes = int(next_prefetch_bytes)  # L2 prefetch of the following GEMV's weights
        self.allreduce = allreduce
        # Tensor parallelism: after the (non-advancing) local head, head_hook(advance)
        # turns the rank's argmax into the global greedy token.
        self.head_hook = head_hook
        if mode not in ("auto", "persistent", "flow", "barrier", "plan"):
            raise ValueError(f"unknown mode {mode!r}")
        self.tp_rank, self.tp_size = tp_rank, tp_size
        # Head: greedy argmax (temperature 0) or a sample of softmax(logits /
        # temperature) -- the reference's sample() without top_k
        # (generate.py:46-63), drawn with counter-based noise keyed by
        # sample_seed and the token position.
        if not (temperature >= 0.0 and math.isfinite(temperature)):
            raise ValueError(f"temperature must be finite and >= 0, got {temperature}")
        self.temperature, self.sample_seed = float(temperature), int(sample_seed)
        self.vocab_offset = int(vocab_offset)
        Hq, Hkv = local_heads if local_heads is not None else (c.n_head, c.n_local_heads)
        self.Hq, self.Hkv, self.D = Hq, Hkv, c.head_dim
        self.max_seq_length = int(max_seq_length)
        S = self.max_seq_length
        f16 = dict(device=dev, dtype=torch.float16)
        i64 = dict(device=dev, dtype=torch.int64)
        dim = c.dim
        qkv_rows = (Hq + 2 * Hkv) * c.head_dim
        ffn0 = model.layers[0].ffn
        inter_local = _linear_segment(getattr(ffn0, "w1", None) or ffn0.gate_proj)["rows"]

        with torch.cuda.device(dev):
            # Device scalars driving the step.
            self.token_in = torch.zeros(1, **i64)
            self.token_out = torch.zeros(1, **i64)
            self.pos = torch.zeros(1, **i64)
            self.history = torch.zeros(max(1, history_len), **i64)
            # Activations (one token).
            self.x_emb = torch.zeros(dim, **f16)
            self.x_buf = torch.zeros(dim, **f16)  # residual stream after attention input
            self.h_buf = torch.zeros(dim, **f16)  # residual stream after MLP input
            self.qkv = torch.zeros(qkv_rows, **f16)
            self.y_attn = torch.zeros(Hq * c.head_dim, **f16)
            self.y_o = torch.zeros(dim, **f16)
            self.act = torch.zeros(inter_local, **f16)
            self.y_down = torch.zeros(dim, **f16)
            head_w = model.output_weight
            self.vocab_local = head_w.shape[0]
            self.logits = torch.zeros(self.vocab_local, **f16)
            self.amax_val = torch.zeros(ARGMAX_CAPACITY, device=dev, dtype=torch.float32)
            self.amax_idx = torch.zeros(ARGMAX_CAPACITY, device=dev, dtype=torch.int32)
            self.amax_counter = torch.zeros(1, device=dev, dtype=torch.int32)
            # KV cache [L, Hkv, S, D] and RoPE table [S, D/2, 2].
            self.k_cache = torch.zeros((c.n_layer, Hkv, S, c.head_dim), **f16)
            self.v_cache = torch.zeros((c.n_layer, Hkv, S, c.head_dim), **f16)
            self.rope = precompute_rope_table(S, c.head_dim, c.rope_base, torch.float16, c.rope_scaling,
                                              c.rope_style).to(dev)
            # fp16 copies of small parameters the kernels read.
            self._keep: List[torch.Tensor] = []
            self._plan = ctypes.c_void_p()
            _lib.check(_lib.lib().nms_plan_create(ctypes.byref(self._plan)), "nms_plan_create")
            self.cut_points: List[int] = []  # plan indices after which an all-reduce runs
            self.gemv_records: List[dict] = []
            self._pending: List[tuple] = []  # launches in step order, added to the plan by _finalize
            self._build(model, attn_splits)
            self._steps = {}
            self.mode = "plan"
            layer_bytes = sum(r["bytes"] for r in self.gemv_records if not r["argmax"]) / max(1, c.n_layer)
            if mode == "auto" and auto_executor(layer_bytes) == "plan":
                mode = "plan"
            if mode != "plan" and allreduce is None and head_hook is None:
                # Persistent executors, in order of preference: the dataflow
                # kernel (no grid barriers), then the barrier kernel.
                kinds = {"auto": FLOW_DEFAULT + ["barrier"], "persistent": FLOW_DEFAULT + ["barrier"],
                         "flow": ["flow"], "barrier": ["barrier"]}[mode]
                for kind in kinds:
                    try:
                        self._create_steps(kind)
                        self.mode = "flow" if kind == "flow" else "persistent"
                        break
                    except NotImplementedError:
                        self._destroy_steps()
                        if kind == kinds[-1] and mode != "auto":
                            raise

    def _create_steps(self, kind: str) -> None:
        """Persistent steps (fixed and advancing head) of the given kernel kind."""
        create = _lib.lib().nms_step_create_flow if kind == "flow" else _lib.lib().nms_step_create
        fixed = list(range(self._head_index)) + [self._head_index]
        adv = list(range(self._head_index)) + [self._head_index + 1]
        for key, recs in ((False, fixed), (True, adv)):
            arr = (ctypes.c_int32 * len(recs))(*recs)
            h = ctypes.c_void_p()
            _lib.check(create(self._plan, arr, len(recs), ctypes.byref(h)), f"nms_step_create ({kind})")
            self._steps[key] = h

    # ------------------------------------------------------------------ build
    def _h(self, t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if t is None:
            return None
        t = t.detach().to(device=self.device, dtype=torch.float16).contiguous()
        self._keep.append(t)
        return t

    def _flags(self, dense: bool = False) -> int:
        return (_lib.NMS_FLAG_PDL if self.pdl else 0) | (_lib.NMS_FLAG_DENSE if dense else 0)

    def _add_gemv(self, linears, *, x, out, x2=None, norm=None, eps=0.0, resid_out=None, swiglu=False,
                  argmax=False, advance=False, x_token=None):
        segs = [_linear_segment(l) for l in linears]
        s0 = segs[0]
        for s in segs[1:]:
            if (s["K"], s["w"], s["w_pad"], s["n"], s["m"], s["dense"]) != (s0["K"], s0["w"], s0["w_pad"], s0["n"],
                                                                          s0["m"], s0["dense"]):
                raise ValueError("fused segments must share K, N:M pattern and packed stride")
        a = _lib.NmsGemvFusedArgs()
        for i, s in enumerate(segs):
            a.seg[i].packed = s["packed"].data_ptr()
            a.seg[i].mat_index = None if s["idx"] is None else s["idx"].data_ptr()
            a.seg[i].rows = s["rows"]
        a.nseg = len(segs)
        a.epilogue = _lib.NMS_EPI_SWIGLU if swiglu else (_lib.NMS_EPI_ARGMAX if argmax else _lib.NMS_EPI_STORE)
        a.prologue = _lib.NMS_PRO_RESID_RMSNORM if norm is not None else _lib.NMS_PRO_PLAIN
        a.flags = self._flags(s0["dense"])
        a.K, a.w, a.w_pad = s0["K"], s0["w"], s0["w_pad"]
        a.block_width, a.vec_width = s0["n"], s0["m"]
        a.x = x.data_ptr()
        if x_token is not None:  # x is a table; the input is row *x_token
            a.x_token = x_token.data_ptr()
            a.x_rows = x.shape[0]
        a.x2 = None if x2 is None else x2.data_ptr()
        a.norm_weight = None if norm is None else norm.data_ptr()
        a.eps = float(eps)
        a.resid_out = None if resid_out is None else resid_out.data_ptr()
        a.out = out.data_ptr()
        a.prefetch_bytes = self.prefetch_bytes
        if argmax:
            a.amax_val = self.amax_val.data_ptr()
            a.amax_idx = self.amax_idx.data_ptr()
            a.amax_counter = self.amax_counter.data_ptr()
            a.token_out = self.token_out.data_ptr()
            a.amax_capacity = ARGMAX_CAPACITY
            a.temperature = self.temperature
            a.sample_seed = self.sample_seed & 0xFFFFFFFFFFFFFFFF
            a.sample_pos = self.pos.data_ptr()
            a.sample_row_offset = self.vocab_offset
            if advance:
                a.next_token = self.token_in.data_ptr()
                a.pos = self.pos.data_ptr()
                a.token_history = self.history.data_ptr()
                a.history_len = self.history.numel()
        self._pending.append(("gemv", a, segs))
        # Algorithmic bytes of this launch: kept values, mask offsets, the
        # input vector(s) and the output (the roofline's traffic model).
        bytes_ = sum(s["rows"] * s["w"] * 2 + (0 if s["dense"] else s["w"]) for s in segs)
        bytes_ += s0["K"] * 2 * (2 if x2 is not None else 1) + (segs[0]["rows"] if swiglu else
                                                               sum(s["rows"] for s in segs)) * 2
        if not argmax or not advance:
            self.gemv_records.append(dict(args=a, bytes=bytes_, dense=s0["dense"], argmax=argmax,
                                          shape=(sum(s["rows"] for s in segs), s0["K"])))

    def step_bytes(self, ctx: int) -> dict:
        """Algorithmic HBM bytes of one decode step at context length `ctx`:
        every GEMV's kept weights, mask offsets, input and output vectors
        (the head once), plus the attention's K/V reads of `ctx` cached
        positions and its K/V writes of the new one, per layer."""
        gemv = sum(r["bytes"] for r in self.gemv_records)
        layers = self.config.n_layer
        kv_read = layers * 2 * self.Hkv * ctx * self.D * 2
        kv_write = layers * 2 * self.Hkv * self.D * 2
        return {"gemv": gemv, "kv": kv_read + kv_write, "total": gemv + kv_read + kv_write}

    def gemv_plan(self, include_head: bool = False):
        """A separate plan holding only this step's GEMV launches (same
        weights and arguments, in step order), for timing the GEMV kernel."""
        plan = ctypes.c_void_p()
        _lib.check(_lib.lib().nms_plan_create(ctypes.byref(plan)))
        total = 0
        for r in self.gemv_records:
            if r["argmax"] and not include_head:
                continue
            _lib.check(_lib.lib().nms_plan_add_gemv(plan, ctypes.byref(r["args"])))
            total += r["bytes"]
        return plan, total

    def _build(self, model: Transformer, attn_splits: int):
        c = self.config
        L = _lib.lib()
        emb = model.tok_embeddings.weight
        if emb.dtype != torch.float16:
            raise TypeError("model must be float16 (the reference decode path is fp16)")
        self.emb = emb
        # The token embedding is folded into the first q/k/v GEMV's prologue
        # (input = row token_in of the embedding table).
        for li, blk in enumerate(model.layers):
            attn, ffn = blk.attn, blk.ffn
            qkv_lins = [attn.wqkv] if c.attn_layout == "fused" else [attn.q_proj, attn.k_proj, attn.v_proj]
            self._add_gemv(qkv_lins, x=emb if li == 0 else self.h_buf, x2=None if li == 0 else self.y_down,
                           norm=self._h(blk.norm1.weight), eps=blk.norm1.eps, resid_out=self.x_buf, out=self.qkv,
                           x_token=self.token_in if li == 0 else None)
            aa = _lib.NmsAttentionArgs()
            aa.qkv = self.qkv.data_ptr()
            aa.k_cache = self.k_cache[li].data_ptr()
            aa.v_cache = self.v_cache[li].data_ptr()
            aa.rope = self.rope.data_ptr()
            qn = self._h(attn.q_norm.weight) if getattr(attn, "q_norm", None) is not None else None
            kn = self._h(attn.k_norm.weight) if getattr(attn, "k_norm", None) is not None else None
            aa.q_norm = None if qn is None else qn.data_ptr()
            aa.k_norm = None if kn is None else kn.data_ptr()
            aa.pos = self.pos.data_ptr()
            aa.y = self.y_attn.data_ptr()
            aa.Hq, aa.Hkv, aa.D, aa.S_max = self.Hq, self.Hkv, c.head_dim, self.max_seq_length
            aa.rope_style = _lib.NMS_ROPE_INTERLEAVED if c.rope_style == "interleaved" else _lib.NMS_ROPE_HALF
            aa.splits = attn_splits
            aa.norm_eps = float(attn.q_norm.eps) if qn is not None else 0.0
            aa.scale = 1.0 / math.sqrt(c.head_dim)
            aa.flags = self._flags()
            self._pending.append(("attn", aa, None))
            o_lin = attn.wo if c.attn_layout == "fused" else attn.o_proj
            self._add_gemv([o_lin], x=self.y_attn, out=self.y_o)
            self.cut_points.append(len(self._pending))
            gate, up, down = ((ffn.w1, ffn.w3, ffn.w2) if c.attn_layout == "fused"
                              else (ffn.gate_proj, ffn.up_proj, ffn.down_proj))
            self._add_gemv([gate, up], x=self.x_buf, x2=self.y_o, norm=self._h(blk.norm2.weight), eps=blk.norm2.eps,
                           resid_out=self.h_buf, out=self.act, swiglu=True)
            self._add_gemv([down], x=self.act, out=self.y_down)
            self.cut_points.append(len(self._pending))
        self._head_index = len(self._pending)
        self._final_norm = self._h(model.norm.weight)
        self._head_args = dict(x=self.h_buf, x2=self.y_down, norm=self._final_norm, eps=model.norm.eps,
                               out=self.logits, argmax=True)
        head = _HeadLinear(model.output_weight)
        self._add_gemv([head], advance=False, **self._head_args)
        self._add_gemv([head], advance=True, **self._head_args)  # variant used by generate()
        self._finalize()

    def _finalize(self) -> None:
        """Give every launch the weight ranges of the GEMV that follows it
        (the head's successor is the next step's first GEMV) for the
        cross-launch L2 prefetch, then add the launches to the plan."""
        L = _lib.lib()
        sms = _lib.num_sms()
        gemv_at = [i for i, e in enumerate(self._pending) if e[0] == "gemv"]
        for i, (kind, a, segs) in enumerate(self._pending):
            nxt = next((j for j in gemv_at if j > i and j != self._head_index + 1), None)
            if nxt is None or (i >= self._head_index):
                nxt = gemv_at[0]
            if kind != "emb" and self.next_prefetch_bytes > 0:
                nsegs = self._pending[nxt][2][:2]
                if kind == "gemv":
                    nb = 2 * sms
                else:
                    nb = a.Hkv * (a.splits if a.splits > 0 else min(16, -(-sms // a.Hkv)))
                head = -(-self.next_prefetch_bytes // (nb * len(nsegs)))
                head = (head + 15) // 16 * 16
                for r, sg in enumerate(nsegs):
                    a.next_prefetch[r] = sg["packed"].data_ptr()
                    a.next_prefetch_bytes[r] = sg["rows"] * sg["w_pad"] * 2
                a.next_prefetch_head = head
            if kind == "gemv":
                _lib.check(L.nms_plan_add_gemv(self._plan, ctypes.byref(a)), "nms_plan_add_gemv")
            elif kind == "attn":
                _lib.check(L.nms_plan_add_attention(self._plan, ctypes.byref(a)), "nms_plan_add_attention")
            else:
                _lib.check(L.nms_plan_add_embedding(self._plan, *a), "nms_plan_add_embedding")
        self._keep_args = self._pending
        self._pending = []

    def size(self) -> int:
        n = ctypes.c_int32()
        _lib.check(_lib.lib().nms_plan_size(self._plan, ctypes.byref(n)))
        return int(n.value)

    # ------------------------------------------------------------------- run
    def _launch(self, begin: int, end: int, stream) -> None:
        if end > begin:
            _lib.check(_lib.lib().nms_plan_launch(self._plan, begin, end, stream.cuda_stream), "nms_plan_launch")

    def step(self, advance: bool = False, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue one decode step: reads token_in and pos on the device,
        writes logits and token_out (and with ``advance`` also token_in,
        history[pos] and pos += 1)."""
        stream = stream or torch.cuda.current_stream(self.device)
        if self.mode in ("persistent", "flow"):
            _lib.check(_lib.lib().nms_step_launch(self._steps[advance], stream.cuda_stream), "nms_step_launch")
            return
        if self.mode == "persistent_tp":
            # One persistent launch: the all-reduces and the vocabulary-
            # parallel greedy token run inside it (tp.TensorParallel.enable_persistent).
            _lib.check(_lib.lib().nms_step_launch(self._steps[advance], stream.cuda_stream), "nms_step_launch")
            return
        begin = 0
        if self.allreduce is not None:
            # Cut points alternate: after the o-projection (partial y_o) and
            # after the down-projection (partial y_down) of every layer.
            for i, cut in enumerate(self.cut_points):
                self._launch(begin, cut, stream)
                with torch.cuda.stream(stream):
                    self.allreduce(self.y_o if i % 2 == 0 else self.y_down)
                begin = cut
        head = self._head_index + (1 if advance and self.head_hook is None else 0)
        self._launch(begin, self._head_index, stream)
        self._launch(head, head + 1, stream)
        if self.head_hook is not None:
            with torch.cuda.stream(stream):
                self.head_hook(advance)

    def check_device(self) -> None:
        """Raise ``RuntimeError`` if a kernel of this library recorded a
        device error (a bounded wait that ran out, a position outside the KV
        cache, or a host abort request), after the work enqueued so far has
        finished.  The steps since the error are void.  The error word is
        cleared and the persistent step's barrier and attention counters are
        zeroed first, so the next step starts clean."""
        code = _lib.device_error(clear=True)
        if code == 0:
            return
        stream = torch.cuda.current_stream(self.device)
        for h in self._steps.values():
            _lib.check(_lib.lib().nms_step_reset(h, stream.cuda_stream), "nms_step_reset")
        self.amax_counter.zero_()  # the head's arrival counter, if the step stopped inside it
        torch.cuda.synchronize(self.device)
        raise RuntimeError(f"decode step failed on the device: error {code} ({DEVICE_ERRORS.get(code, 'unknown')}); "
                           "the steps since the last check are void")

    def prefill(self, tokens, start_pos: int = 0) -> torch.Tensor:
        """Batched prefill: run ``tokens`` at positions ``start_pos ..`` through
        the model's own layers in one pass -- every N:M projection as one
        tensor-core GEMM over all the tokens (``nmsparse::gemm_packed``, the
        same sparse weights the decode steps use), attention by
        ``F.scaled_dot_product_attention`` under the causal mask -- writing
        K/V straight into this engine's caches.  Leaves ``pos`` at the next
        position and ``token_in`` at the greedy next token, so a decode step
        continues from there.  Returns the last token's logits (fp16 [vocab]).

        The reference prefills through a dense ``F.linear`` with the unpruned
        weights (src/spmv/nmsparse_linear.py:55-68) or token by token through
        the decode path (NM_DECODE_ONLY=1); this is the sparse batched form."""
        if self.tp_size != 1:
            raise NotImplementedError("batched prefill runs on one GPU; a tensor-parallel engine takes the prompt "
                                      "through its decode step")
        toks = torch.as_tensor(list(tokens), dtype=torch.int64).to(self.device)
        T = int(toks.numel())
        if T == 0:
            raise ValueError("prefill needs at least one token")
        if start_pos < 0 or start_pos + T > self.max_seq_length:
            raise ValueError(f"positions [{start_pos}, {start_pos + T}) outside the cache of {self.max_seq_length}")
        m = self.model
        saved = [blk.attn.kv_cache for blk in m.layers]
        try:
            for li, blk in enumerate(m.layers):
                blk.attn.kv_cache = _CacheView(self.k_cache[li:li + 1], self.v_cache[li:li + 1])
            with torch.no_grad(), torch.cuda.device(self.device), sparse_prefill():
                input_pos = torch.arange(start_pos, start_pos + T, device=self.device)
                rope = self.rope[input_pos]
                x = m.tok_embeddings(toks.view(1, T))
                for blk in m.layers:
                    x = blk(x, input_pos, rope)
                x = m.norm(x[:, -1:])
                logits = F.linear(x, m.output_weight).view(-1)
                nxt = torch.argmax(logits).view(1)
                self.pos.fill_(start_pos + T)
                self.token_in.copy_(nxt)
                if start_pos + T - 1 < self.history.numel():
                    self.history[start_pos + T - 1: start_pos + T].copy_(nxt)
        finally:
            for blk, kv in zip(m.layers, saved):
                blk.attn.kv_cache = kv
        return logits

    def reset(self) -> None:
        self.k_cache.zero_()
        self.v_cache.zero_()
        self.pos.zero_()
        self.token_in.zero_()
        self.history.zero_()

    def fill_synthetic_cache(self, ctx: int, std: float = 0.02, seed: int = 0) -> None:
        """Reference fixed-context protocol: KV cache ~ N(0, std), position ctx
        (bench_llama_3_8b_fp16_fixed_ptx.py:145-152)."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        for t in (self.k_cache, self.v_cache):
            t.normal_(0.0, std, generator=g)
        self.pos.fill_(ctx)

    def capture(self, advance: bool = False, warmup: int = 3) -> torch.cuda.CUDAGraph:
        """CUDA graph of one decode step (side-stream warm-up, then capture)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        pos0 = self.pos.clone()
        tok0 = self.token_in.clone()
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.step(advance=advance, stream=s)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.pos.copy_(pos0)
        self.token_in.copy_(tok0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step(advance=advance, stream=s)
        torch.cuda.synchronize(self.device)
        return g

    def step_timeline(self, advance: bool = False, warmup: int = 2, detail: bool = False,
                      sm_mhz: float = 1965.0) -> dict:
        """Run the persistent step once with its timeline enabled and return
        per-stage statistics in microseconds: work (previous barrier release to
        the slowest CTA's finish), imbalance (slowest - fastest CTA finish) and
        barrier (slowest finish to release).  With ``detail`` each stage also
        gets ``marks_us``: for each detail mark 1..6 of the kernel's trace
        (GEMV: input staged, norm statistic, masks ready, gathered vector,
        items consumed, finish; attention: q/k/v prepared at mark 4,
        published at 5, finish at 6) the mean over the CTAs that recorded it
        of the time since stage entry, counted in SM clock cycles and
        converted at ``sm_mhz`` (None where no CTA recorded it)."""
        if self.mode not in ("persistent", "persistent_tp", "flow"):
            raise RuntimeError("the timeline needs a persistent executor")
        L = _lib.lib()
        h = self._steps[advance]
        ns, grid = ctypes.c_int32(), ctypes.c_int32()
        _lib.check(L.nms_step_info(h, ctypes.byref(ns), ctypes.byref(grid)))
        n, g = int(ns.value), int(grid.value)
        base = 1 + n * (g + 1)
        marks = 8
        buf = torch.zeros(base + (n * g * marks if detail else 0), dtype=torch.int64, device=self.device)
        for _ in range(warmup):
            self.step(advance=advance)
        _lib.check(L.nms_step_set_trace(h, buf.data_ptr(), buf.numel()))
        self.step(advance=advance)
        torch.cuda.synchronize(self.device)
        _lib.check(L.nms_step_set_trace(h, None, 0))
        t = buf.cpu().double()
        t0 = t[0].item()
        rows = t[1:base].view(n, g + 1)
        det = t[base:].view(n, g, marks) if detail else None
        stages = []
        prev = t0
        for s in range(n):
            fin = rows[s, :g]
            # The flow kernel has no barrier: a stage "releases" when its
            # slowest CTA finishes.
            rel = rows[s, g].item() if (s + 1 < n and rows[s, g].item() > 0) else fin.max().item()
            st = {"work_us": (fin.max().item() - prev) / 1e3, "imbalance_us": (fin.max() - fin.min()).item() / 1e3,
                  "barrier_us": (rel - fin.max().item()) / 1e3}
            if det is not None:
                d = det[s]
                e = d[:, 0]
                mk = []
                for k in range(1, 7):
                    ok = d[:, k] > 0  # CTAs that recorded the mark (attention: CTAs with a unit)
                    mk.append((d[ok, k] - e[ok]).mean().item() / sm_mhz if bool(ok.any()) else None)
                st["marks_us"] = mk
            stages.append(st)
            prev = rel
        return {"total_us": (prev - t0) / 1e3, "stages": stages}

    def _destroy_steps(self) -> None:
        for h in getattr(self, "_steps", {}).values():
            _lib.lib().nms_step_destroy(h)
        self._steps = {}

    def close(self) -> None:
        self._destroy_steps()
        if self._plan:
            _lib.lib().nms_plan_destroy(self._plan)
            self._plan = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _HeadLinear:
    """Dense output head adapter (tied or untied weight)."""

    def __init__(self, weight: torch.Tensor):
        self.weight = weight


class _CacheView(nn.Module):
    """KV-cache update onto one layer of the engine's caches ([1, Hkv, S, D]
    views), for the model's eager attention during a batched prefill."""

    def __init__(self, k: torch.Tensor, v: torch.Tensor):
        super().__init__()
        self.k, self.v = k, v

    def update(self, input_pos, k_val, v_val):
        self.k[:, :, input_pos] = k_val
        self.v[:, :, input_pos] = v_val
        return self.k, self.v
