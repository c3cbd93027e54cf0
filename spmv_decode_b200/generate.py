"""Generation API over the fused decode engine (mirrors generate.py).

* ``decode_one_token(engine, token, input_pos)`` -- one step, returns the
  greedy next token and the logits (generate.py:80-91; greedy instead of the
  exponential-race sample, generate.py:46-63).
* ``decode_n_tokens`` / ``generate`` -- the decode loop (generate.py:93-119,
  176-247) as replays of one captured CUDA graph whose head kernel writes
  the next input token and advances the position on the device, so the loop
  needs no host synchronisation.  Prompt tokens are fed one per step through
  the same decode path (prefill in decode-only mode, which every reference
  benchmark uses: NM_DECODE_ONLY=1), or with ``batched_prefill=True`` all
  at once through ``DecodeEngine.prefill`` (sparse tensor-core GEMMs).
* ``build_model`` -- a Transformer for a named configuration with N:M
  sparse (or dense) linears; ``init="reference"`` reproduces the reference
  packer bit for bit, ``init="device"`` draws the same distributions on the
  GPU in seconds for multi-GB models.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .engine import DecodeEngine
from .model import ModelArgs, Transformer
from .nmsparse_linear import swap_to_nmsparse


def decode_one_token(engine: DecodeEngine, token: int, input_pos: int) -> Tuple[int, torch.Tensor]:
    """Eager single step at position ``input_pos``; returns (token, logits)."""
    engine.token_in.fill_(int(token))
    engine.pos.fill_(int(input_pos))
    engine.step(advance=False)
    tok = int(engine.token_out.item())
    engine.check_device()
    return tok, engine.logits.clone()


class GraphDecoder:
    """A captured decode step (advancing) plus the host loop around it."""

    def __init__(self, engine: DecodeEngine):
        self.engine = engine
        self.graph = engine.capture(advance=True)

    def replay(self) -> None:
        self.graph.replay()

    def run(self, prompt: Sequence[int], max_new_tokens: int, start_pos: int = 0,
            keep_logits: bool = False) -> Tuple[List[int], Optional[torch.Tensor]]:
        """Feed ``prompt`` from ``start_pos`` then generate ``max_new_tokens``
        greedy tokens; returns (generated tokens, optional logits per step)."""
        e = self.engine
        n_prompt = len(prompt)
        total = n_prompt + max_new_tokens - 1
        if start_pos + total > e.max_seq_length or start_pos + total > e.history.numel():
            raise ValueError("sequence exceeds the engine's max_seq_length / history buffer")
        prompt_dev = torch.tensor(list(prompt), dtype=torch.int64, device=e.device)
        e.pos.fill_(start_pos)
        logits = []
        for i in range(total):
            if i < n_prompt:
                e.token_in.copy_(prompt_dev[i: i + 1])
            self.graph.replay()
            if keep_logits:
                logits.append(e.logits.clone())
        torch.cuda.synchronize(e.device)
        e.check_device()
        first = start_pos + n_prompt - 1
        toks = e.history[first: first + max_new_tokens].tolist()
        return toks, (torch.stack(logits) if keep_logits else None)


def generate(engine: DecodeEngine, prompt: Sequence[int], max_new_tokens: int, *,
             batched_prefill: bool = False) -> List[int]:
    """Greedy generation through a captured decode step (generate.py:176-247).

    ``batched_prefill=True`` first runs all prompt tokens but the last through
    ``engine.prefill`` (one sparse tensor-core GEMM per projection for the
    whole prompt) instead of one decode step per prompt token."""
    prompt = list(prompt)
    if batched_prefill and len(prompt) > 1:
        engine.prefill(prompt[:-1])
        return GraphDecoder(engine).run(prompt[-1:], max_new_tokens, start_pos=len(prompt) - 1)[0]
    return GraphDecoder(engine).run(prompt, max_new_tokens)[0]


def decode_n_tokens(engine: DecodeEngine, cur_token: int, input_pos: int, num_new_tokens: int) -> List[int]:
    """generate.py:93-119: continue from ``cur_token`` at ``input_pos``."""
    return GraphDecoder(engine).run([cur_token], num_new_tokens, start_pos=input_pos)[0]


def build_model(name_or_args, *, nm: Optional[Tuple[int, int]] = (32, 64), device="cuda", seed: int = 0,
                init: str = "device", std: float = 0.02) -> Transformer:
    """Transformer with random-init embeddings/head ~ N(0, std), unit norms and
    N:M sparse linears (``nm=(n, m)``, 50% as in the reference) or dense
    linears ~ N(0, std) (``nm=None``), all fp16 on ``device``.  Built on the
    meta device first, so no dense weight of a sparse model is materialised."""
    args = name_or_args if isinstance(name_or_args, ModelArgs) else ModelArgs.from_name(name_or_args)
    device = torch.device(device)
    with torch.device("meta"):
        model = Transformer(args)
    gen = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        t = torch.empty(shape, dtype=torch.float16, device=device)
        # draw in chunks to bound the fp32 temporary
        flat = t.view(-1)
        step = 1 << 26
        for i in range(0, flat.numel(), step):
            j = min(flat.numel(), i + step)
            flat[i:j] = (torch.randn(j - i, generator=gen, device=device) * std).to(torch.float16)
        return t

    model.tok_embeddings = nn.Embedding(args.vocab_size, args.dim, device="meta")
    model.tok_embeddings.weight = nn.Parameter(randn(args.vocab_size, args.dim), requires_grad=False)
    if model.output is not None:
        model.output.weight = nn.Parameter(randn(args.vocab_size, args.dim), requires_grad=False)
    for mod in model.modules():
        if mod.__class__.__name__ == "RMSNorm":
            mod.weight = nn.Parameter(torch.ones(mod.weight.shape, dtype=torch.float16, device=device),
                                      requires_grad=False)
    if nm is not None:
        n, m = nm
        if 2 * n != m:
            raise ValueError("the reference packer keeps M/2 of every M (50% sparsity)")
        swap_to_nmsparse(model, m, device, seed=seed, init=init, keep_dense=False)
    else:
        for blk in model.layers:
            for sub in (blk.attn, blk.ffn):
                for name, lin in list(sub.named_children()):
                    if isinstance(lin, nn.Linear):
                        new = nn.Linear(lin.in_features, lin.out_features, bias=False, device="meta")
                        new.weight = nn.Parameter(randn(lin.out_features, lin.in_features), requires_grad=False)
                        setattr(sub, name, new)
    return model
