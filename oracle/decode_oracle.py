"""ORACLE -- test infrastructure, not product code (see oracle/__init__.py).

torch-CPU restatement of the reference decode step, with the same fp16
rounding points:

* gpt-fast path (model.py): Transformer.forward :159-170, TransformerBlock
  :185-188, Attention :215-245 (fused wqkv split, RoPE on (2i, 2i+1) pairs
  in fp32 from the fp16 table, KV update, causal GQA attention), FeedForward
  :255-256, RMSNorm :259-270, precompute_freqs_cis :295-307 incl. Llama-3.1
  scaling :273-292.
* HF Qwen3 path (the reference's Qwen3 benchmarks): q_norm/k_norm per head
  before RoPE, rotate_half RoPE with fp16 rounding per op, tied embeddings.
* Sparse linears: nmsparse::gemv semantics -- fp32 accumulation of
  fp16 x fp16, result rounded to fp16 (triton_spmv.py:81-115, 318) --
  computed as the masked dense matrix times the vector in fp32.
* Greedy token = argmax of the fp16 logits (lowest index on ties).

``make_sparse_ref`` restates the reference packer
(src/spmv/nmsparse_linear.py:14-33, shared-mask branch) so fixtures can be
rebuilt from seeds; tests/test_oracle_golden.py pins it.

Pinned by tests/test_decode_oracle.py against tests/golden/decode_*.npz,
which the reference decode path itself produced.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch


def make_sparse_ref(K: int, N: int, M: int, seed: int):
    """(mat_data [w, N] fp16, mat_index [K/M, M/2] uint8) of the reference packer."""
    nnz = M // 2
    nb = K // M
    w = nb * nnz
    g = torch.Generator().manual_seed(seed)
    mat_data = (torch.randn(w, N, generator=g, dtype=torch.float32) / (K ** 0.5)).to(torch.float16)
    mat_index = torch.empty(nb, nnz, dtype=torch.uint8)
    for bank in range(nb):
        mat_index[bank] = torch.randperm(M, generator=g)[:nnz].sort().values.to(torch.uint8)
    return mat_data, mat_index


def masked_dense_t(mat_data: torch.Tensor, mat_index: torch.Tensor, K: int, M: int) -> torch.Tensor:
    """[N, K] fp16 dense matrix of a shared-mask layer (microbench:145-164)."""
    w, h = mat_data.shape
    nb, nnz = mat_index.shape
    cols = (torch.arange(nb)[:, None] * M + mat_index.long()).reshape(-1)
    dense = torch.zeros((h, K), dtype=torch.float16)
    dense[:, cols] = mat_data.t()
    return dense


def rope_table(seq_len: int, head_dim: int, base: float, rope_scaling: Optional[dict], style: str) -> torch.Tensor:
    """[S, D/2, 2] fp16 (cos, sin): model.py:295-307 (interleaved) or the HF
    rotary embedding (half)."""
    freqs = 1.0 / (base ** (torch.arange(0, head_dim, 2)[: (head_dim // 2)].float() / head_dim))
    if rope_scaling is not None:
        factor = rope_scaling["factor"]
        lo, hi = rope_scaling["low_freq_factor"], rope_scaling["high_freq_factor"]
        old = rope_scaling["original_max_position_embeddings"]
        lo_w, hi_w = old / lo, old / hi
        out = []
        for f in freqs:
            wl = 2 * math.pi / f
            if wl < hi_w:
                out.append(f)
            elif wl > lo_w:
                out.append(f / factor)
            else:
                sm = (old / wl - lo) / (hi - lo)
                out.append((1 - sm) * f / factor + sm * f)
        freqs = torch.tensor(out, dtype=freqs.dtype)
    t = torch.arange(seq_len)
    if style == "interleaved":
        ang = torch.outer(t, freqs)
        cis = torch.polar(torch.ones_like(ang), ang)
        tab = torch.stack([cis.real, cis.imag], dim=-1)
    else:
        ang = t.float()[:, None] * freqs[None, :]
        tab = torch.stack([ang.cos(), ang.sin()], dim=-1)
    return tab.to(torch.float16)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = (xf * torch.rsqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + eps)).to(torch.float16)
    return y * w


def rope_apply(x: torch.Tensor, rope_row: torch.Tensor, style: str) -> torch.Tensor:
    """x [H, D] fp16, rope_row [D/2, 2] fp16."""
    if style == "interleaved":
        xs = x.float().reshape(x.shape[0], -1, 2)
        c, s = rope_row[:, 0].float(), rope_row[:, 1].float()
        out = torch.stack([xs[..., 0] * c - xs[..., 1] * s, xs[..., 1] * c + xs[..., 0] * s], -1)
        return out.flatten(1).to(torch.float16)
    cos = torch.cat([rope_row[:, 0], rope_row[:, 0]])
    sin = torch.cat([rope_row[:, 1], rope_row[:, 1]])
    half = x.shape[-1] // 2
    rot = torch.cat([-x[:, half:], x[:, :half]], dim=-1)
    return (x * cos) + (rot * sin)


@dataclass
class OracleLayer:
    qkv: List[torch.Tensor]  # dense [rows, K] fp16 matrices (1 fused or 3 split)
    wo: torch.Tensor
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    norm1: torch.Tensor
    norm2: torch.Tensor
    q_norm: Optional[torch.Tensor]
    k_norm: Optional[torch.Tensor]


class OracleModel:
    """Batch-1 decode of a decoder with dense (masked) fp16 weights on the CPU."""

    def __init__(self, *, layers: List[OracleLayer], emb: torch.Tensor, head: torch.Tensor, final_norm: torch.Tensor,
                 n_head: int, n_kv: int, head_dim: int, eps: float, rope: torch.Tensor, style: str,
                 max_seq: int, linear_dtype=torch.float32):
        self.layers, self.emb, self.head, self.final_norm = layers, emb, head, final_norm
        self.n_head, self.n_kv, self.D, self.eps = n_head, n_kv, head_dim, eps
        self.rope, self.style = rope, style
        self.linear_dtype = linear_dtype
        if linear_dtype == torch.float32:
            # Convert once; every step multiplies the same matrices.
            for L in self.layers:
                L.qkv = [W.float() for W in L.qkv]
                L.wo, L.gate, L.up, L.down = L.wo.float(), L.gate.float(), L.up.float(), L.down.float()
            self.head = self.head.float()
        self.k = [torch.zeros(n_kv, max_seq, head_dim, dtype=torch.float16) for _ in layers]
        self.v = [torch.zeros(n_kv, max_seq, head_dim, dtype=torch.float16) for _ in layers]
        # Tensor-parallel shard: sums the fp16 partial o- and down-projection
        # outputs over the ranks (identity on one rank).
        self.reduce = None

    # -- construction --------------------------------------------------------
    @classmethod
    def from_transformer(cls, model, max_seq: Optional[int] = None, linear_dtype=torch.float32,
                         heads: Optional[tuple] = None):
        """Copy the weights of a spmv_decode_b200 Transformer (sparse linears
        expanded to masked dense matrices via their reference-layout values).
        ``heads`` = (query heads, KV heads) of a tensor-parallel shard."""
        c = model.config

        def dense(lin):
            if hasattr(lin, "mat_index"):
                return masked_dense_t(lin.reference_mat_data().cpu(), lin.mat_index.cpu(), lin.in_features,
                                      lin.vec_width)
            return lin.weight.detach().cpu().to(torch.float16)

        layers = []
        for blk in model.layers:
            a, f = blk.attn, blk.ffn
            if c.attn_layout == "fused":
                qkv = [dense(a.wqkv)]
                wo = dense(a.wo)
                gate, up, down = dense(f.w1), dense(f.w3), dense(f.w2)
            else:
                qkv = [dense(a.q_proj), dense(a.k_proj), dense(a.v_proj)]
                wo = dense(a.o_proj)
                gate, up, down = dense(f.gate_proj), dense(f.up_proj), dense(f.down_proj)
            qn = a.q_norm.weight.detach().cpu().half() if getattr(a, "q_norm", None) is not None else None
            kn = a.k_norm.weight.detach().cpu().half() if getattr(a, "k_norm", None) is not None else None
            layers.append(OracleLayer(qkv, wo, gate, up, down, blk.norm1.weight.detach().cpu().half(),
                                      blk.norm2.weight.detach().cpu().half(), qn, kn))
        S = max_seq or 64
        return cls(layers=layers, emb=model.tok_embeddings.weight.detach().cpu().half(),
                   head=model.output_weight.detach().cpu().half(), final_norm=model.norm.weight.detach().cpu().half(),
                   n_head=heads[0] if heads else c.n_head, n_kv=heads[1] if heads else c.n_local_heads,
                   head_dim=c.head_dim, eps=c.norm_eps,
                   rope=rope_table(max(S, 8), c.head_dim, c.rope_base, c.rope_scaling, c.rope_style),
                   style=c.rope_style, max_seq=S, linear_dtype=linear_dtype)

    @classmethod
    def from_golden(cls, z, kind: str):
        """Rebuild the model of a decode fixture (tests/golden/decode_*.npz):
        embeddings/head/norms from the file, sparse linears from the seeds."""
        vocab, n_layer, n_head, n_kv, dim, inter, M, seed, prompt_len, steps = (int(v) for v in z["cfg"])
        D = 128
        emb = torch.from_numpy(z["emb"]).view(torch.float16)
        if kind == "llama":
            head = torch.from_numpy(z["head"]).view(torch.float16)
            eps, style = 1e-5, "interleaved"
            scaling = dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                           original_max_position_embeddings=8192)
            shapes = [("wqkv", (n_head + 2 * n_kv) * D, dim), ("wo", dim, n_head * D), ("w1", inter, dim),
                      ("w3", inter, dim), ("w2", dim, inter)]
        else:
            head = emb
            eps, style, scaling = float(z["eps"][0]), "half", None
            shapes = [("q", n_head * D, dim), ("k", n_kv * D, dim), ("v", n_kv * D, dim), ("o", dim, n_head * D),
                      ("gate", inter, dim), ("up", inter, dim), ("down", dim, inter)]
        cnt = 0
        layers = []
        for li in range(n_layer):
            w = {}
            for name, N, K in shapes:
                md, mi = make_sparse_ref(K, N, M, seed + cnt)
                w[name] = masked_dense_t(md, mi, K, M)
                cnt += 1
            ones = torch.ones(dim, dtype=torch.float16)
            if kind == "llama":
                layers.append(OracleLayer([w["wqkv"]], w["wo"], w["w1"], w["w3"], w["w2"], ones, ones, None, None))
            else:
                f16 = lambda a: torch.from_numpy(a).view(torch.float16)  # noqa: E731
                layers.append(OracleLayer([w["q"], w["k"], w["v"]], w["o"], w["gate"], w["up"], w["down"],
                                          f16(z["in_norm"][li]), f16(z["post_norm"][li]), f16(z["q_norm"][li]),
                                          f16(z["k_norm"][li])))
        final = (torch.from_numpy(z["final_norm"]).view(torch.float16) if kind == "qwen3"
                 else torch.ones(dim, dtype=torch.float16))
        S = prompt_len + steps + 8
        return cls(layers=layers, emb=emb, head=head, final_norm=final, n_head=n_head, n_kv=n_kv, head_dim=D,
                   eps=eps, rope=rope_table(256, D, float(z["rope_base"][0]), scaling, style), style=style,
                   max_seq=S)

    # -- math ----------------------------------------------------------------
    def _linear(self, W: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        if self.linear_dtype == torch.float16:
            return torch.nn.functional.linear(x.view(1, -1), W).view(-1)
        return (W @ x.float()).to(torch.float16)

    def step(self, token: int, pos: int) -> torch.Tensor:
        """Logits (fp16 [vocab]) of one decode step at position ``pos``."""
        D, Hq, Hkv = self.D, self.n_head, self.n_kv
        G = Hq // Hkv
        x = self.emb[token].clone()
        rope_row = self.rope[pos]
        for li, L in enumerate(self.layers):
            xn = rmsnorm(x, L.norm1, self.eps)
            qkv = torch.cat([self._linear(W, xn) for W in L.qkv])
            q = qkv[: Hq * D].view(Hq, D)
            k = qkv[Hq * D: (Hq + Hkv) * D].view(Hkv, D)
            v = qkv[(Hq + Hkv) * D:].view(Hkv, D)
            if L.q_norm is not None:
                q = rmsnorm(q, L.q_norm, self.eps)
                k = rmsnorm(k, L.k_norm, self.eps)
            q = rope_apply(q, rope_row, self.style)
            k = rope_apply(k, rope_row, self.style)
            self.k[li][:, pos] = k
            self.v[li][:, pos] = v
            Kc = self.k[li][:, : pos + 1].float()  # [Hkv, P, D]
            Vc = self.v[li][:, : pos + 1].float()
            qf = q.float().view(Hkv, G, D)
            s = torch.einsum("hgd,hpd->hgp", qf, Kc) / math.sqrt(D)
            p = torch.softmax(s, dim=-1)
            y = torch.einsum("hgp,hpd->hgd", p, Vc).reshape(Hq * D).to(torch.float16)
            o = self._linear(L.wo, y)
            if self.reduce is not None:
                o = self.reduce(o)
            x = x + o
            hn = rmsnorm(x, L.norm2, self.eps)
            g = self._linear(L.gate, hn)
            u = self._linear(L.up, hn)
            act = torch.nn.functional.silu(g.float()).to(torch.float16) * u
            dn = self._linear(L.down, act)
            if self.reduce is not None:
                dn = self.reduce(dn)
            x = x + dn
        xn = rmsnorm(x, self.final_norm, self.eps)
        return self._linear(self.head, xn)

    def greedy(self, prompt: List[int], steps: int):
        """Token-by-token prefill then greedy decode; returns (tokens, logits per position)."""
        logits_all, tokens = [], []
        cur = int(prompt[0])
        for pos in range(len(prompt) + steps):
            lg = self.step(cur, pos)
            logits_all.append(lg)
            nxt = int(torch.argmax(lg).item())
            if pos + 1 < len(prompt):
                cur = int(prompt[pos + 1])
            else:
                tokens.append(nxt)
                cur = nxt
        return tokens, torch.stack(logits_all)


def _masked_random(rows: int, K: int, m: Optional[int], std: float, gen: torch.Generator) -> torch.Tensor:
    """Dense fp16 [rows, K] ~ N(0, std) with a shared 50% in-group mask
    (all rows keep the same m/2 columns of every group of m), or unmasked
    when m is None."""
    W = (torch.randn(rows, K, generator=gen) * std).to(torch.float16)
    if m is not None:
        keys = torch.rand(K // m, m, generator=gen)
        drop = keys.argsort(dim=1)[:, m // 2:]
        cols = (torch.arange(K // m)[:, None] * m + drop).reshape(-1)
        W[:, cols] = 0
    return W


def cpu_decode_sample(config, nm: Optional[tuple], ctx: int, sample_layers: int = 2, steps: int = 3,
                      threads: Optional[int] = None, seed: int = 0, warmup: int = 1,
                      single_thread_steps: int = 0) -> dict:
    """Time the reference's torch CPU decode path on a bounded sample of a
    workload: ``sample_layers`` decoder layers of the configuration's shapes
    plus the full output head, dense masked fp16 weights multiplied with
    F.linear (the reference's CPU path, microbench_triton_torchmv.py:210-211),
    KV cache ~ N(0, 0.02) of length ``ctx``.  The per-token time of the whole
    model is extrapolated as n_layer * (layer time) + head time.
    ``single_thread_steps`` > 0 also times that many steps of the same sample
    on one host thread (``single_thread_ms_per_token``)."""
    import time

    if threads:
        torch.set_num_threads(threads)
    c = config
    D = c.head_dim
    m = None if nm is None else nm[1]
    gen = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(sample_layers):
        qkv_rows = (c.n_head + 2 * c.n_local_heads) * D
        ones = torch.ones(c.dim, dtype=torch.float16)
        qn = torch.ones(D, dtype=torch.float16) if c.qk_norm else None
        layers.append(OracleLayer([_masked_random(qkv_rows, c.dim, m, 0.02, gen)],
                                  _masked_random(c.dim, c.n_head * D, m, 0.02, gen),
                                  _masked_random(c.intermediate_size, c.dim, m, 0.02, gen),
                                  _masked_random(c.intermediate_size, c.dim, m, 0.02, gen),
                                  _masked_random(c.dim, c.intermediate_size, m, 0.02, gen), ones, ones, qn, qn))
    emb = (torch.randn(c.vocab_size, c.dim, generator=gen) * 0.02).to(torch.float16)
    head = emb if c.tie_embeddings else (torch.randn(c.vocab_size, c.dim, generator=gen) * 0.02).to(torch.float16)
    om = OracleModel(layers=layers, emb=emb, head=head, final_norm=torch.ones(c.dim, dtype=torch.float16),
                     n_head=c.n_head, n_kv=c.n_local_heads, head_dim=D, eps=c.norm_eps,
                     rope=rope_table(ctx + steps + 2, D, c.rope_base, c.rope_scaling, c.rope_style),
                     style=c.rope_style, max_seq=ctx + steps + 2, linear_dtype=torch.float16)
    for kc, vc in zip(om.k, om.v):
        kc.normal_(0, 0.02, generator=gen)
        vc.normal_(0, 0.02, generator=gen)
    x = torch.randn(c.dim, generator=gen).to(torch.float16)
    for _ in range(max(1, warmup)):  # untimed warm-up steps
        om.step(123, ctx)
        om._linear(om.head, x)
    def timed(n):
        t_step, t_head = [], []
        for i in range(n):
            t0 = time.perf_counter()
            om.step(123, ctx)
            t1 = time.perf_counter()
            om._linear(om.head, x)
            t2 = time.perf_counter()
            t_step.append(t1 - t0)
            t_head.append(t2 - t1)
        step_s = sorted(t_step)[len(t_step) // 2]
        head_s = sorted(t_head)[len(t_head) // 2]
        return max(step_s - head_s, 0.0) / sample_layers, head_s

    layer_s, head_s = timed(steps)
    used = torch.get_num_threads()
    single = None
    if single_thread_steps > 0:
        torch.set_num_threads(1)
        try:
            om.step(123, ctx)  # one untimed step on the single thread
            l1, h1 = timed(single_thread_steps)
            single = 1e3 * (c.n_layer * l1 + h1)
        finally:
            torch.set_num_threads(used)
    return {
        "ms_per_token": 1e3 * (c.n_layer * layer_s + head_s),
        "single_thread_ms_per_token": single,
        "layer_ms": 1e3 * layer_s,
        "head_ms": 1e3 * head_s,
        "threads": used,
        "sample": f"{sample_layers} of {c.n_layer} decoder layers + full output head, ctx {ctx}, "
                  f"median of {steps} steps, dense masked fp16 F.linear; per-token time = "
                  f"{c.n_layer} x layer + head",
    }
