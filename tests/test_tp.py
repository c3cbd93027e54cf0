"""Tensor-parallel decode (spmv_decode_b200/tp.py) on the CPU.

* Shards reassemble the full model: row shards of q/k/v, gate/up and the
  head concatenate to the full matrices, column shards of the o- and
  down-projections (whole mask groups, re-padded) concatenate along K.
* The decomposition is exact up to fp16 rounding of partial sums: two gloo
  ranks each run the decode oracle on their shard, sum the o- and
  down-projection partials with an all-reduce, and pick the greedy token with
  the same candidate all-gather + global_argmax the GPU engine captures; the
  result is compared with the single-process oracle on the full model.
  Tolerance: logits within 2e-2 x max|logit| (fp16 partial sums), and the
  same greedy tokens.
"""
import copy
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.decode_oracle import OracleModel
from spmv_decode_b200.model import ModelArgs, Transformer
from spmv_decode_b200.nmsparse_linear import swap_to_nmsparse
from spmv_decode_b200.tp import global_argmax, gather_candidates, shard_model

TOL = 2e-2
PROMPT = [3, 17, 250, 9]
STEPS = 6


def _tiny(seed=0, layout="fused"):
    if layout == "fused":
        args = ModelArgs(block_size=64, vocab_size=512, n_layer=2, n_head=4, n_local_heads=2, dim=256,
                         intermediate_size=512)
    else:
        args = ModelArgs(block_size=64, vocab_size=512, n_layer=2, n_head=4, n_local_heads=2, dim=256, head_dim=128,
                         intermediate_size=512, rope_style="half", qk_norm=True, tie_embeddings=True,
                         attn_layout="split")
    torch.manual_seed(seed)
    model = Transformer(args)
    with torch.no_grad():
        model.tok_embeddings.weight.normal_(0, 0.5)
        if model.output is not None:
            model.output.weight.normal_(0, 0.05)
    model = model.half()
    swap_to_nmsparse(model, 32, "cpu", seed=seed)
    return model


def _dense(lin):
    if hasattr(lin, "mat_index"):
        return lin.dense_masked_weight()
    return lin.weight.detach()


@pytest.mark.parametrize("layout", ["fused", "split"])
def test_shards_reassemble_the_model(layout):
    full = _tiny(layout=layout)
    world = 2
    shards = []
    for r in range(world):
        m = copy.deepcopy(full)
        shards.append((m, shard_model(m, world, r)))
    c = full.config
    for li, blk in enumerate(full.layers):
        a, f = blk.attn, blk.ffn
        if layout == "fused":
            D, Hq, Hkv = c.head_dim, c.n_head, c.n_local_heads
            W = _dense(a.wqkv)
            q, k, v = W[: Hq * D], W[Hq * D: (Hq + Hkv) * D], W[(Hq + Hkv) * D:]
            parts = [_dense(m.layers[li].attn.wqkv) for m, _ in shards]
            hq, hkv = Hq // world * D, Hkv // world * D
            assert torch.equal(torch.cat([p[:hq] for p in parts]), q)
            assert torch.equal(torch.cat([p[hq: hq + hkv] for p in parts]), k)
            assert torch.equal(torch.cat([p[hq + hkv:] for p in parts]), v)
            pairs = [("wo", 1), ("w1", 0), ("w3", 0), ("w2", 1)]
            mods = [(a, "wo"), (f, "w1"), (f, "w3"), (f, "w2")]
        else:
            pairs = [("q_proj", 0), ("k_proj", 0), ("v_proj", 0), ("o_proj", 1), ("gate_proj", 0), ("up_proj", 0),
                     ("down_proj", 1)]
            mods = [(a, n) for n, _ in pairs[:4]] + [(f, n) for n, _ in pairs[4:]]
        for (owner, name), (_, dim) in zip(mods, pairs):
            whole = _dense(getattr(owner, name))
            sub = [m.layers[li].attn if owner is a else m.layers[li].ffn for m, _ in shards]
            got = torch.cat([_dense(getattr(s, name)) for s in sub], dim=dim)
            assert torch.equal(got, whole), (li, name)
    head = torch.cat([m.output_weight.detach() for m, _ in shards])
    assert torch.equal(head, full.output_weight.detach())
    assert shards[1][1].vocab_offset == c.vocab_size // world


def test_global_argmax_breaks_ties_like_torch_argmax():
    logits = torch.tensor([0.5, 2.0, -1.0, 2.0, 2.0, 0.0])
    world = 3
    cands = []
    for r in range(world):
        part = logits[r * 2:(r + 1) * 2]
        i = int(torch.argmax(part))
        cands.append([float(part[i]), float(r * 2 + i)])
    tok = global_argmax(torch.tensor(cands))
    assert int(tok) == int(torch.argmax(logits)) == 1


def _rank_main(rank, world, port, layout, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        model = _tiny(layout=layout)
        info = shard_model(model, world, rank)
        om = OracleModel.from_transformer(model, max_seq=32, heads=info.local_heads)

        def reduce(t):
            s = t.float()
            dist.all_reduce(s)
            return s.to(torch.float16)

        om.reduce = reduce
        cur, toks, logits_all = PROMPT[0], [], []
        for pos in range(len(PROMPT) + STEPS):
            local = om.step(cur, pos)
            parts = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(parts, local)
            logits_all.append(torch.cat(parts))
            i = int(torch.argmax(local))
            cand = torch.tensor([float(local[i]), float(info.vocab_offset + i)])
            nxt = int(global_argmax(gather_candidates(cand, world)))
            if pos + 1 < len(PROMPT):
                cur = PROMPT[pos + 1]
            else:
                toks.append(nxt)
                cur = nxt
        if rank == 0:
            out.put((toks, torch.stack(logits_all)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["fused", "split"])
def test_two_gloo_ranks_match_single_process_oracle(layout):
    ref_toks, ref_logits = OracleModel.from_transformer(_tiny(layout=layout), max_seq=32).greedy(PROMPT, STEPS)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, layout, q)) for r in range(2)]
    for p in procs:
        p.start()
    toks, logits = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    err = (logits.float() - ref_logits.float()).abs().amax(dim=1)
    scale = ref_logits.float().abs().amax(dim=1)
    assert bool((err <= TOL * scale).all()), (err / scale).max().item()
    assert toks == ref_toks
