"""Tensor-parallel batch-1 decode: one process per GPU over NCCL.

The reference runs decode on one GPU (its gpt-fast ``model.py`` keeps the
``tp.py`` hooks of its upstream but ships no tensor-parallel module).  This
module splits the same model Megatron-style so a step streams 1/N of the
weights per GPU:

* q/k/v and gate/up are split by output rows (whole query / KV heads, whole
  intermediate rows); the embedding table and the norms are replicated;
* the o- and down-projections are split by input columns in whole mask
  groups (M columns), so every shard is itself a shared-mask N:M matrix with
  the matching rows of ``mat_index``; their partial outputs are summed either
  inside the persistent step kernel (fp32 partials written into every rank's
  exchange area over NVLink, summed in rank order) or, with the plan executor,
  by an NCCL all-reduce of fp16 partials captured in the step's CUDA graph;
* the output head is split by vocabulary rows; every rank takes the argmax of
  its logits (first index on ties, as ``torch.argmax``), the (value, index)
  candidates are all-gathered, and the global greedy token is the largest
  value with the smallest index -- the same token ``argmax`` over the full
  logits gives.

Sharding works on CPU modules too (the multi-process tests run it with the
gloo backend against the decode oracle); the engine itself needs the CUDA
library.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Optional, Tuple

import torch
import torch.distributed as dist
from torch import nn

from .nmsparse_linear import NmSparseLinear
from .nmsparse_op import packed_row_stride


class DenseShard(nn.Module):
    """A dense fp16 weight slice (rows of an nn.Linear / the output head)."""

    def __init__(self, weight: torch.Tensor):
        super().__init__()
        self.weight = nn.Parameter(weight.contiguous(), requires_grad=False)

    def forward(self, x):
        return torch.nn.functional.linear(x, self.weight)


def _sparse_like(packed: torch.Tensor, mat_index: torch.Tensor, K: int, N: int, M: int) -> NmSparseLinear:
    lin = NmSparseLinear(N, K, M, 0, packed.device, init="empty", layout="shared")
    lin.mat_data = packed.contiguous()
    lin.mat_index = mat_index.contiguous()
    lin.w = mat_index.shape[0] * mat_index.shape[1]
    lin.h = N
    return lin


def _shared_only(lin: NmSparseLinear) -> None:
    if lin.layout != "shared":
        raise NotImplementedError("tensor-parallel shards are built from shared-mask layers; "
                                  "per-row (layout='rowwise') layers are not sharded")


def shard_rows(lin: nn.Module, ranges) -> nn.Module:
    """Rows ``ranges`` ([(r0, r1), ...], concatenated in order) of a linear."""
    if isinstance(lin, NmSparseLinear):
        _shared_only(lin)
        packed = torch.cat([lin.mat_data[r0:r1] for r0, r1 in ranges])
        return _sparse_like(packed, lin.mat_index, lin.in_features, packed.shape[0], lin.vec_width)
    return DenseShard(torch.cat([lin.weight.detach()[r0:r1] for r0, r1 in ranges]))


def shard_cols(lin: nn.Module, k0: int, k1: int) -> nn.Module:
    """Input columns [k0, k1) of a linear; for a sparse one [k0, k1) must be
    whole mask groups, and the shard keeps their compressed columns and
    mask rows (re-padded to the packed row stride)."""
    if isinstance(lin, NmSparseLinear):
        _shared_only(lin)
        M, n = lin.vec_width, lin.block_width
        if k0 % M or k1 % M:
            raise ValueError(f"column shard [{k0}, {k1}) is not made of whole {M}-column mask groups")
        g0, g1 = k0 // M, k1 // M
        w = (g1 - g0) * n
        packed = torch.zeros((lin.h, packed_row_stride(w)), dtype=lin.mat_data.dtype, device=lin.mat_data.device)
        packed[:, :w] = lin.mat_data[:, g0 * n: g1 * n]
        return _sparse_like(packed, lin.mat_index[g0:g1], k1 - k0, lin.h, M)
    return DenseShard(lin.weight.detach()[:, k0:k1])


@dataclasses.dataclass
class ShardInfo:
    world: int
    rank: int
    local_heads: Tuple[int, int]  # (query heads, KV heads) of this rank
    vocab_offset: int
    vocab_local: int


def shard_model(model, world: int, rank: int) -> ShardInfo:
    """Replace ``model``'s linears by this rank's shards, in place."""
    c = model.config
    D = c.head_dim
    Hq, Hkv, inter = c.n_head, c.n_local_heads, c.intermediate_size
    if Hkv % world or Hq % world:
        raise ValueError(f"{Hq} query / {Hkv} KV heads do not split over {world} ranks")
    if inter % world or c.vocab_size % world:
        raise ValueError(f"intermediate size {inter} / vocabulary {c.vocab_size} do not split over {world} ranks")
    hq, hkv, il = Hq // world, Hkv // world, inter // world
    q0, k0 = rank * hq * D, rank * hkv * D
    for blk in model.layers:
        attn, ffn = blk.attn, blk.ffn
        if c.attn_layout == "fused":
            attn.wqkv = shard_rows(attn.wqkv, [(q0, q0 + hq * D), (Hq * D + k0, Hq * D + k0 + hkv * D),
                                               ((Hq + Hkv) * D + k0, (Hq + Hkv) * D + k0 + hkv * D)])
            attn.wo = shard_cols(attn.wo, q0, q0 + hq * D)
            ffn.w1 = shard_rows(ffn.w1, [(rank * il, (rank + 1) * il)])
            ffn.w3 = shard_rows(ffn.w3, [(rank * il, (rank + 1) * il)])
            ffn.w2 = shard_cols(ffn.w2, rank * il, (rank + 1) * il)
        else:
            attn.q_proj = shard_rows(attn.q_proj, [(q0, q0 + hq * D)])
            attn.k_proj = shard_rows(attn.k_proj, [(k0, k0 + hkv * D)])
            attn.v_proj = shard_rows(attn.v_proj, [(k0, k0 + hkv * D)])
            attn.o_proj = shard_cols(attn.o_proj, q0, q0 + hq * D)
            ffn.gate_proj = shard_rows(ffn.gate_proj, [(rank * il, (rank + 1) * il)])
            ffn.up_proj = shard_rows(ffn.up_proj, [(rank * il, (rank + 1) * il)])
            ffn.down_proj = shard_cols(ffn.down_proj, rank * il, (rank + 1) * il)
    vl = c.vocab_size // world
    model.output = DenseShard(model.output_weight.detach()[rank * vl:(rank + 1) * vl])
    return ShardInfo(world, rank, (hq, hkv), rank * vl, vl)


def global_argmax(cand: torch.Tensor) -> torch.Tensor:
    """Greedy token from the ranks' candidates ``cand`` [world, 2] = (max
    logit, its global index) as fp32: the largest value, smallest index on
    ties (``torch.argmax`` over the concatenated logits).  Graph-capturable."""
    vals, idx = cand[:, 0], cand[:, 1]
    best = vals.max()
    pick = torch.where(vals == best, idx, torch.full_like(idx, float("inf")))
    return pick.min().to(torch.int64).view(1)


def gather_candidates(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather every rank's [2] candidate into [world, 2]."""
    out = torch.empty((world, 2), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(-1), local, group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, local, group=group)
    return out


class TensorParallel:
    """Collectives of one rank's decode step: NCCL (captured in the graph)
    for the plan executor and the head; with :meth:`enable_persistent` the
    o-/down-projection all-reduces run inside the persistent step kernel over
    NVLink peer memory."""

    def __init__(self, info: ShardInfo, device: torch.device, group=None):
        self.info, self.group = info, group
        self.device = device
        self.cand = torch.zeros(2, dtype=torch.float32, device=device)
        self._own_area = None
        self._peer_areas = []

    def enable_persistent(self, engine) -> None:
        """Give ``engine`` persistent steps (fixed and advancing) over all its
        stages: exchange points after every o- and down-projection write
        partial rows into every rank's exchange area, and the vocabulary-
        parallel head swaps its (logit, index) candidates the same way.  One
        cudaMalloc'd area per rank, mapped into the other processes through
        CUDA IPC handles swapped with an all-gather.  Raises
        NotImplementedError if the step does not fit."""
        from . import _lib

        lib = _lib.lib()
        w, r = self.info.world, self.info.rank
        steps = {}
        try:
            for adv in (False, True):
                recs = list(range(engine._head_index)) + [engine._head_index + (1 if adv else 0)]
                arr = (ctypes.c_int32 * len(recs))(*recs)
                st = ctypes.c_void_p()
                _lib.check(lib.nms_step_create(engine._plan, arr, len(recs), ctypes.byref(st)), "nms_step_create")
                steps[adv] = st
            nreduce, dim = len(engine.cut_points), engine.config.dim
            nbytes = lib.nms_tp_area_bytes(nreduce, w, dim)
            own = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            with torch.cuda.device(self.device):
                _lib.check(lib.nms_ipc_alloc(nbytes, ctypes.byref(own), handle), "nms_ipc_alloc")
            self._own_area = own
            handles = [None] * w
            dist.all_gather_object(handles, handle.raw, group=self.group)
            areas = []
            for k in range(w):
                if k == r:
                    areas.append(own.value)
                    continue
                p = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _lib.check(lib.nms_ipc_open(ctypes.create_string_buffer(handles[k], 64), ctypes.byref(p)),
                               "nms_ipc_open")
                self._peer_areas.append(p)
                areas.append(p.value)
            cfg = _lib.NmsTpConfig()
            cfg.world, cfg.rank, cfg.dim, cfg.vocab_offset = w, r, dim, self.info.vocab_offset
            for k, a in enumerate(areas):
                cfg.area[k] = a
            stages = [c - 1 for c in engine.cut_points]
            sarr = (ctypes.c_int32 * len(stages))(*stages)
            for st in steps.values():
                _lib.check(lib.nms_step_set_tp(st, sarr, len(stages), ctypes.byref(cfg)), "nms_step_set_tp")
        except Exception:
            for st in steps.values():
                lib.nms_step_destroy(st)
            self.close()
            raise
        engine._steps.update(steps)
        engine.mode = "persistent_tp"

    def close(self) -> None:
        """Unmap the peers' exchange areas and free this rank's (after every
        rank is done with them)."""
        from . import _lib

        if self._own_area is None and not self._peer_areas:
            return
        lib = _lib.lib()
        torch.cuda.synchronize(self.device)
        if dist.is_initialized():
            dist.barrier(group=self.group)
        for p in self._peer_areas:
            lib.nms_ipc_close(p)
        self._peer_areas = []
        if self._own_area is not None:
            lib.nms_ipc_free(self._own_area)
            self._own_area = None

    def allreduce(self, t: torch.Tensor) -> None:
        dist.all_reduce(t, group=self.group)

    def head_hook(self, engine, advance: bool) -> None:
        """After the local head: global greedy token into token_out (and
        with ``advance`` into token_in, history[pos], pos += 1, as the
        single-GPU head's generation hooks do)."""
        val = engine.logits.index_select(0, engine.token_out).float()
        self.cand[0:1].copy_(val)
        self.cand[1:2].copy_((engine.token_out + self.info.vocab_offset).float())
        tok = global_argmax(gather_candidates(self.cand, self.info.world, self.group))
        engine.token_out.copy_(tok)
        if advance:
            hist = engine.history
            p = engine.pos.clamp(0, hist.numel() - 1)
            hist.index_copy_(0, p, tok)
            engine.token_in.copy_(tok)
            engine.pos.add_(1)


def build_tp_engine(cfg, nm: Optional[Tuple[int, int]], world: int, rank: int, device: torch.device, *,
                    max_seq: int, seed: int = 0, prefetch_bytes: int = 0, next_prefetch_bytes: int = 0,
                    history_len: int = 0, group=None, mode: str = "auto", temperature: float = 0.0,
                    sample_seed: int = 0):
    """This rank's decode engine for ``cfg`` (the same weights as the
    single-GPU model built with ``seed``), and its TensorParallel state.
    ``mode``: "plan" (NCCL all-reduces between launches), "persistent"
    (all-reduces inside the persistent step over NVLink) or "auto"
    (persistent when it fits).  ``temperature`` > 0 samples the token (the
    same draw as one GPU: the noise is keyed by the global vocabulary row);
    it needs the persistent executor, whose exchange compares the sampling
    keys."""
    if temperature > 0 and mode == "plan":
        raise NotImplementedError("temperature sampling under tensor parallelism needs the persistent executor")
    from .engine import DecodeEngine
    from .generate import build_model

    model = build_model(cfg, nm=nm, device=device, seed=seed, init="device")
    info = shard_model(model, world, rank)
    torch.cuda.empty_cache()
    tp = TensorParallel(info, device, group)
    eng = DecodeEngine(model, max_seq, prefetch_bytes=prefetch_bytes, next_prefetch_bytes=next_prefetch_bytes,
                       history_len=history_len, mode="plan", allreduce=tp.allreduce, tp_rank=rank, tp_size=world,
                       local_heads=info.local_heads, head_hook=lambda adv: tp.head_hook(eng, adv),
                       temperature=temperature, sample_seed=sample_seed, vocab_offset=info.vocab_offset)
    if mode in ("auto", "persistent"):
        try:
            tp.enable_persistent(eng)
        except NotImplementedError:
            if mode == "persistent" or temperature > 0:
                raise
    return eng, tp
