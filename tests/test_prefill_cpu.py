"""The model's multi-token forward -- the layer path DecodeEngine.prefill runs
on the GPU with sparse GEMMs -- against the oracle's token-by-token decode, on
the CPU.

Each sparse linear is given its dense equivalent (the kept values scattered
to their columns) as the dense weight, so F.linear computes the same product
the sparse GEMM does; the whole prompt then goes through one forward (causal
attention over the KV cache at positions 0..T-1).  The logits at every
position must be within 2e-2 x max|logit| of the oracle's decode step at that
position (the decode tests' bar), for the gpt-fast and the HF Qwen3 block
layouts.
"""
import pytest
import torch

from oracle.decode_oracle import OracleModel
from spmv_decode_b200.model import ModelArgs, Transformer
from spmv_decode_b200.nmsparse_linear import NmSparseLinear, swap_to_nmsparse

TOL = 2e-2
PROMPT = [3, 17, 250, 9, 77, 400, 5, 123, 64, 301]


def _tiny(layout):
    if layout == "fused":
        args = ModelArgs(block_size=64, vocab_size=512, n_layer=2, n_head=4, n_local_heads=2, dim=256,
                         intermediate_size=512)
    else:
        args = ModelArgs(block_size=64, vocab_size=512, n_layer=2, n_head=4, n_local_heads=2, dim=256, head_dim=128,
                         intermediate_size=512, rope_style="half", qk_norm=True, tie_embeddings=True,
                         attn_layout="split")
    torch.manual_seed(0)
    model = Transformer(args)
    with torch.no_grad():
        model.tok_embeddings.weight.normal_(0, 0.5)
        if model.output is not None:
            model.output.weight.normal_(0, 0.05)
    model = model.half()
    swap_to_nmsparse(model, 32, "cpu", seed=0, keep_dense=False)
    for mod in model.modules():
        if isinstance(mod, NmSparseLinear):
            mod.weight = mod.dense_masked_weight()
    return model


@pytest.mark.parametrize("layout", ["fused", "split"])
def test_multi_token_forward_matches_token_by_token_oracle(layout):
    torch.set_num_threads(4)
    model = _tiny(layout)
    om = OracleModel.from_transformer(model, max_seq=32)
    ref = torch.stack([om.step(tok, pos) for pos, tok in enumerate(PROMPT)]).float()
    model.setup_caches(1, 32)
    T = len(PROMPT)
    with torch.no_grad():
        logits = model(None, torch.tensor([PROMPT]), torch.arange(T)).float()[0]
    err = (logits - ref).abs().amax(dim=1)
    scale = ref.abs().amax(dim=1)
    assert bool((err <= TOL * scale).all()), (err / scale).max().item()
