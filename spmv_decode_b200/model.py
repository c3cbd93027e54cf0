# Portions of this file (find_multiple, the ModelArgs fields, __post_init__,
# from_name and the transformer_configs table, KVCache.update, RMSNorm,
# apply_rope_scaling and the frequency lines of the RoPE table) follow
# gpt-fast's model.py, which the reference ships as model.py under this notice:
#
#   Copyright (c) Meta Platforms, Inc. and affiliates.
#   All rights reserved.
#
#   This source code is licensed under the license found in the
#   LICENSE file in the root directory of this source tree.
#
# (gpt-fast is distributed under the BSD 3-Clause License.)  They are kept
# alike on purpose: state dicts, configuration names and the bit-identical
# fp16 RoPE table that decode parity needs depend on them.
"""Decoder model definitions for the decode engine (gpt-fast compatible).

Mirrors the reference's model.py (ModelArgs, KVCache, Transformer,
TransformerBlock, Attention, FeedForward, RMSNorm, RoPE; model.py:43-322)
and extends it to the shapes the reference benchmarks through HF
transformers (Qwen3: head_dim independent of dim, per-head q/k RMSNorm,
rotate-half RoPE, tied embeddings).  Two block layouts:

* ``attn_layout="fused"`` -- gpt-fast names: ``attention.wqkv / wo``,
  ``feed_forward.w1 / w3 / w2``, ``attention_norm / ffn_norm``
  (model.py:177-256).
* ``attn_layout="split"`` -- HF names: ``self_attn.q_proj / k_proj /
  v_proj / o_proj (+ q_norm / k_norm)``, ``mlp.gate_proj / up_proj /
  down_proj``, ``input_layernorm / post_attention_layernorm``.

``swap_to_nmsparse`` (nmsparse_linear.py) walks either layout in the same
order as the reference, so seeds match.  ``Transformer.forward`` is the
plain PyTorch path (single-token steps call the nmsparse op); the fused
sm_100a decode step lives in ``engine.DecodeEngine``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor


def find_multiple(n: int, k: int) -> int:
    if n % k == 0:
        return n
    return n + k - (n % k)


@dataclass
class ModelArgs:
    block_size: int = 2048
    vocab_size: int = 32000
    n_layer: int = 32
    n_head: int = 32
    dim: int = 4096
    intermediate_size: Optional[int] = None
    n_local_heads: int = -1
    head_dim: int = 0  # 0 = dim // n_head (gpt-fast rule, model.py:64)
    rope_base: float = 10000
    norm_eps: float = 1e-5
    rope_scaling: Optional[dict] = None
    # Extensions for the HF Qwen3 architecture.
    rope_style: str = "interleaved"  # "interleaved" (gpt-fast) | "half" (HF rotate_half)
    qk_norm: bool = False
    tie_embeddings: bool = False
    attn_layout: str = "fused"  # "fused" (wqkv) | "split" (q/k/v)

    def __post_init__(self):
        if self.n_local_heads == -1:
            self.n_local_heads = self.n_head
        if self.intermediate_size is None:
            hidden_dim = 4 * self.dim
            n_hidden = int(2 * hidden_dim / 3)
            self.intermediate_size = find_multiple(n_hidden, 256)
        if not self.head_dim:
            self.head_dim = self.dim // self.n_head

    @property
    def q_size(self) -> int:
        return self.n_head * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.n_local_heads * self.head_dim

    @classmethod
    def from_name(cls, name: str):
        if name in transformer_configs:
            return cls(**transformer_configs[name])
        config = [c for c in transformer_configs if c.lower() in str(name).lower()]
        if not config:
            raise KeyError(f"unknown model config {name!r}")
        if len(config) > 1:
            config.sort(key=len, reverse=True)
            assert len(config[0]) != len(config[1]), name
        return cls(**transformer_configs[config[0]])


_LLAMA31_SCALING = dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0, original_max_position_embeddings=8192)

transformer_configs = {
    # gpt-fast table of the reference (model.py:82-105)
    "CodeLlama-7b-Python-hf": dict(block_size=16384, vocab_size=32000, n_layer=32, dim=4096, rope_base=1000000),
    "7B": dict(n_layer=32, n_head=32, dim=4096),
    "13B": dict(n_layer=40, n_head=40, dim=5120),
    "30B": dict(n_layer=60, n_head=52, dim=6656),
    "34B": dict(n_layer=48, n_head=64, dim=8192, vocab_size=32000, n_local_heads=8, intermediate_size=22016,
                rope_base=1000000),
    "70B": dict(n_layer=80, n_head=64, dim=8192, n_local_heads=8, intermediate_size=28672),
    "Mistral-7B": dict(n_layer=32, n_head=32, n_local_heads=8, dim=4096, intermediate_size=14336, vocab_size=32000),
    "stories15M": dict(n_layer=6, n_head=6, dim=288),
    "stories110M": dict(n_layer=12, n_head=12, dim=768),
    "llama-3-8b": dict(block_size=8192, n_layer=32, n_head=32, n_local_heads=8, dim=4096, intermediate_size=14336,
                       vocab_size=128256, rope_base=500000),
    "llama-3-70b": dict(block_size=8192, n_layer=80, n_head=64, n_local_heads=8, dim=8192, intermediate_size=28672,
                        vocab_size=128256, rope_base=500000),
    "llama-3.1-8b": dict(block_size=131072, n_layer=32, n_head=32, n_local_heads=8, dim=4096,
                         intermediate_size=14336, vocab_size=128256, rope_base=500000,
                         rope_scaling=_LLAMA31_SCALING),
    "llama-3.1-70b": dict(block_size=131072, n_layer=80, n_head=64, n_local_heads=8, dim=8192,
                          intermediate_size=28672, vocab_size=128256, rope_base=500000,
                          rope_scaling=_LLAMA31_SCALING),
    "qwen2.5-72b": dict(block_size=131072, n_layer=80, n_head=64, n_local_heads=8, dim=8192,
                        intermediate_size=29568, vocab_size=152064, rope_base=1000000, norm_eps=1e-5),
    "llama-3.1-405b": dict(block_size=131072, n_layer=126, n_head=128, n_local_heads=8, dim=16384,
                           intermediate_size=53248, vocab_size=128256, rope_base=500000,
                           rope_scaling=_LLAMA31_SCALING),
    # HF Qwen3 architectures the reference benchmarks (BASELINE configs 3 and 5)
    "qwen3-0.6b": dict(block_size=40960, n_layer=28, n_head=16, n_local_heads=8, dim=1024, head_dim=128,
                       intermediate_size=3072, vocab_size=151936, rope_base=1000000, norm_eps=1e-6,
                       rope_style="half", qk_norm=True, tie_embeddings=True, attn_layout="split"),
    "qwen3-14b": dict(block_size=40960, n_layer=40, n_head=40, n_local_heads=8, dim=5120, head_dim=128,
                      intermediate_size=17408, vocab_size=151936, rope_base=1000000, norm_eps=1e-6,
                      rope_style="half", qk_norm=True, tie_embeddings=False, attn_layout="split"),
    "qwen3-32b": dict(block_size=40960, n_layer=64, n_head=64, n_local_heads=8, dim=5120, head_dim=128,
                      intermediate_size=25600, vocab_size=151936, rope_base=1000000, norm_eps=1e-6,
                      rope_style="half", qk_norm=True, tie_embeddings=False, attn_layout="split"),
}


class KVCache(nn.Module):
    """Static KV cache [B, H, S, D] (model.py:107-123)."""

    def __init__(self, max_batch_size, max_seq_length, n_heads, head_dim, dtype=torch.float16):
        super().__init__()
        cache_shape = (max_batch_size, n_heads, max_seq_length, head_dim)
        self.register_buffer("k_cache", torch.zeros(cache_shape, dtype=dtype))
        self.register_buffer("v_cache", torch.zeros(cache_shape, dtype=dtype))

    def update(self, input_pos, k_val, v_val):
        assert input_pos.shape[0] == k_val.shape[2]
        k_out = self.k_cache
        v_out = self.v_cache
        k_out[:, :, input_pos] = k_val
        v_out[:, :, input_pos] = v_val
        return k_out, v_out


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) in fp32, cast back, times weight (model.py:259-270)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def _norm(self, x):
        return x * torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + self.eps)

    def forward(self, x: Tensor) -> Tensor:
        output = self._norm(x.float()).type_as(x)
        return output * self.weight


def apply_rope_scaling(freqs: torch.Tensor, rope_scaling: Optional[dict] = None):
    """Llama 3.1 frequency scaling (model.py:273-292)."""
    factor = rope_scaling["factor"]
    low_freq_factor = rope_scaling["low_freq_factor"]
    high_freq_factor = rope_scaling["high_freq_factor"]
    old_context_len = rope_scaling["original_max_position_embeddings"]
    low_freq_wavelen = old_context_len / low_freq_factor
    high_freq_wavelen = old_context_len / high_freq_factor
    new_freqs = []
    for freq in freqs:
        wavelen = 2 * math.pi / freq
        if wavelen < high_freq_wavelen:
            new_freqs.append(freq)
        elif wavelen > low_freq_wavelen:
            new_freqs.append(freq / factor)
        else:
            assert low_freq_wavelen != high_freq_wavelen
            smooth = (old_context_len / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
            new_freqs.append((1 - smooth) * freq / factor + smooth * freq)
    return torch.tensor(new_freqs, dtype=freqs.dtype, device=freqs.device)


def precompute_rope_table(seq_len: int, head_dim: int, base: float, dtype=torch.float16,
                          rope_scaling: Optional[dict] = None, style: str = "interleaved") -> Tensor:
    """[seq_len, head_dim/2, 2] (cos, sin) table in ``dtype``.

    interleaved: precompute_freqs_cis (model.py:295-307) -- polar() of
    outer(t, freqs) in fp32, cast to the model dtype.
    half: HF rotary embedding -- cos/sin of position*inv_freq in fp32, cast
    to the model dtype (attention_scaling 1.0 for default RoPE).
    """
    freqs = 1.0 / (base ** (torch.arange(0, head_dim, 2)[: (head_dim // 2)].float() / head_dim))
    if rope_scaling is not None:
        freqs = apply_rope_scaling(freqs, rope_scaling)
    t = torch.arange(seq_len, device=freqs.device)
    if style == "interleaved":
        ang = torch.outer(t, freqs)
        freqs_cis = torch.polar(torch.ones_like(ang), ang)
        cache = torch.stack([freqs_cis.real, freqs_cis.imag], dim=-1)
    else:
        ang = t.float()[:, None] * freqs[None, :]
        cache = torch.stack([ang.cos(), ang.sin()], dim=-1)
    return cache.to(dtype=dtype)


def apply_rotary_emb(x: Tensor, rope: Tensor, style: str) -> Tensor:
    """x [B, S, H, D]; rope [S, D/2, 2].  Rounding order of the reference
    paths: gpt-fast computes in fp32 and casts once (model.py:310-322); HF
    rotate_half rounds after every fp16 op."""
    if style == "interleaved":
        xs = x.float().reshape(*x.shape[:-1], -1, 2)
        r = rope.view(1, xs.size(1), 1, xs.size(3), 2)
        out = torch.stack([xs[..., 0] * r[..., 0] - xs[..., 1] * r[..., 1],
                           xs[..., 1] * r[..., 0] + xs[..., 0] * r[..., 1]], -1)
        return out.flatten(3).type_as(x)
    cos = torch.cat([rope[..., 0], rope[..., 0]], dim=-1).to(x.dtype)[None, :, None, :]
    sin = torch.cat([rope[..., 1], rope[..., 1]], dim=-1).to(x.dtype)[None, :, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return (x * cos) + (rot * sin)


class Attention(nn.Module):
    """gpt-fast fused-qkv attention (model.py:191-245), with head_dim and
    wo sized n_head*head_dim -> dim."""

    def __init__(self, config: ModelArgs):
        super().__init__()
        total_head_dim = config.q_size + 2 * config.kv_size
        self.wqkv = nn.Linear(config.dim, total_head_dim, bias=False)
        self.wo = nn.Linear(config.q_size, config.dim, bias=False)
        self.kv_cache = None
        self.config = config

    def project_qkv(self, x):
        c = self.config
        return self.wqkv(x).split([c.q_size, c.kv_size, c.kv_size], dim=-1)

    def out_proj(self, y):
        return self.wo(y)


class SplitAttention(nn.Module):
    """HF Qwen3 attention module layout: q/k/v/o projections, q/k RMSNorm."""

    def __init__(self, config: ModelArgs):
        super().__init__()
        self.q_proj = nn.Linear(config.dim, config.q_size, bias=False)
        self.k_proj = nn.Linear(config.dim, config.kv_size, bias=False)
        self.v_proj = nn.Linear(config.dim, config.kv_size, bias=False)
        self.o_proj = nn.Linear(config.q_size, config.dim, bias=False)
        self.q_norm = RMSNorm(config.head_dim, config.norm_eps) if config.qk_norm else None
        self.k_norm = RMSNorm(config.head_dim, config.norm_eps) if config.qk_norm else None
        self.kv_cache = None
        self.config = config

    def project_qkv(self, x):
        return self.q_proj(x), self.k_proj(x), self.v_proj(x)

    def out_proj(self, y):
        return self.o_proj(y)


def _attention_forward(mod, x: Tensor, rope: Tensor, input_pos: Tensor) -> Tensor:
    c = mod.config
    bsz, seqlen, _ = x.shape
    q, k, v = mod.project_qkv(x)
    q = q.view(bsz, seqlen, c.n_head, c.head_dim)
    k = k.view(bsz, seqlen, c.n_local_heads, c.head_dim)
    v = v.view(bsz, seqlen, c.n_local_heads, c.head_dim)
    if getattr(mod, "q_norm", None) is not None:
        q = mod.q_norm(q)
        k = mod.k_norm(k)
    q = apply_rotary_emb(q, rope, c.rope_style)
    k = apply_rotary_emb(k, rope, c.rope_style)
    q, k, v = map(lambda t: t.transpose(1, 2), (q, k, v))
    k, v = mod.kv_cache.update(input_pos, k, v)
    kv_idx = torch.arange(k.shape[-2], device=q.device)
    attn_mask = (kv_idx[None, :] <= input_pos.reshape(-1)[:, None])[None, None]
    y = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, enable_gqa=(c.n_head != c.n_local_heads))
    y = y.transpose(1, 2).contiguous().view(bsz, seqlen, c.q_size)
    return mod.out_proj(y)


class FeedForward(nn.Module):
    """SwiGLU MLP, gpt-fast names (model.py:248-256)."""

    def __init__(self, config: ModelArgs) -> None:
        super().__init__()
        self.w1 = nn.Linear(config.dim, config.intermediate_size, bias=False)
        self.w3 = nn.Linear(config.dim, config.intermediate_size, bias=False)
        self.w2 = nn.Linear(config.intermediate_size, config.dim, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class SplitMLP(nn.Module):
    """SwiGLU MLP, HF names."""

    def __init__(self, config: ModelArgs) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(config.dim, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.dim, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.dim, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class TransformerBlock(nn.Module):
    """h = x + attn(norm(x)); out = h + mlp(norm(h)) (model.py:177-188)."""

    def __init__(self, config: ModelArgs) -> None:
        super().__init__()
        self.config = config
        if config.attn_layout == "fused":
            self.attention = Attention(config)
            self.feed_forward = FeedForward(config)
            self.attention_norm = RMSNorm(config.dim, config.norm_eps)
            self.ffn_norm = RMSNorm(config.dim, config.norm_eps)
        else:
            self.self_attn = SplitAttention(config)
            self.mlp = SplitMLP(config)
            self.input_layernorm = RMSNorm(config.dim, config.norm_eps)
            self.post_attention_layernorm = RMSNorm(config.dim, config.norm_eps)

    # Uniform accessors used by the engine and the eager forward.
    @property
    def attn(self):
        return self.attention if self.config.attn_layout == "fused" else self.self_attn

    @property
    def ffn(self):
        return self.feed_forward if self.config.attn_layout == "fused" else self.mlp

    @property
    def norm1(self):
        return self.attention_norm if self.config.attn_layout == "fused" else self.input_layernorm

    @property
    def norm2(self):
        return self.ffn_norm if self.config.attn_layout == "fused" else self.post_attention_layernorm

    def forward(self, x: Tensor, input_pos: Tensor, rope: Tensor) -> Tensor:
        h = x + _attention_forward(self.attn, self.norm1(x), rope, input_pos)
        return h + self.ffn(self.norm2(h))


class Transformer(nn.Module):
    def __init__(self, config: ModelArgs) -> None:
        super().__init__()
        self.config = config
        self.tok_embeddings = nn.Embedding(config.vocab_size, config.dim)
        self.layers = nn.ModuleList(TransformerBlock(config) for _ in range(config.n_layer))
        self.norm = RMSNorm(config.dim, eps=config.norm_eps)
        self.output = None if config.tie_embeddings else nn.Linear(config.dim, config.vocab_size, bias=False)
        self.rope: Optional[Tensor] = None
        self.max_batch_size = -1
        self.max_seq_length = -1

    @property
    def output_weight(self) -> Tensor:
        return self.tok_embeddings.weight if self.output is None else self.output.weight

    def setup_caches(self, max_batch_size, max_seq_length):
        """Static KV caches and the RoPE table (model.py:141-157)."""
        if self.max_seq_length >= max_seq_length and self.max_batch_size >= max_batch_size:
            return
        c = self.config
        max_seq_length = find_multiple(max_seq_length, 8)
        self.max_seq_length = max_seq_length
        self.max_batch_size = max_batch_size
        dtype = self.tok_embeddings.weight.dtype
        device = self.tok_embeddings.weight.device
        for b in self.layers:
            b.attn.kv_cache = KVCache(max_batch_size, max_seq_length, c.n_local_heads, c.head_dim, dtype).to(device)
        self.rope = precompute_rope_table(c.block_size, c.head_dim, c.rope_base, dtype, c.rope_scaling,
                                          c.rope_style).to(device)

    def forward(self, mask, idx: Tensor, input_pos: Optional[Tensor] = None) -> Tensor:
        """Eager forward (model.py:159-170); ``mask`` is accepted for API
        compatibility and ignored (causal masking from input_pos)."""
        assert self.rope is not None, "Caches must be initialized first"
        rope = self.rope[input_pos]
        x = self.tok_embeddings(idx)
        for layer in self.layers:
            x = layer(x, input_pos, rope)
        x = self.norm(x)
        return F.linear(x, self.output_weight)

    @classmethod
    def from_name(cls, name: str):
        return cls(ModelArgs.from_name(name))
