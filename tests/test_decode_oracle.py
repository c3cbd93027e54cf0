"""Pin the CPU decode oracle to the reference decode path.

tests/golden/decode_*.npz were produced by the reference's own decode code
(gpt-fast model.py and HF Qwen3ForCausalLM with the reference
swap_to_nmsparse and the reference Triton kernel under the interpreter).
The oracle rebuilds the same weights from the stored seeds and tensors and
must reproduce the greedy tokens exactly and the logits within
LOGIT_TOL * max|logit| (fp32 summation order differs from the reference
kernel's atomics, so single fp16 roundings of intermediates may differ)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.decode_oracle import OracleModel, make_sparse_ref
from spmv_decode_b200.nmsparse_linear import make_sparse

LOGIT_TOL = 1e-2


@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_oracle_reproduces_reference_decode(kind):
    z = np.load(GOLDEN / f"decode_{kind}_tiny.npz")
    vocab, n_layer, n_head, n_kv, dim, inter, M, seed, prompt_len, steps = (int(v) for v in z["cfg"])
    om = OracleModel.from_golden(z, kind)
    tokens, logits = om.greedy(z["prompt"].tolist(), steps)
    ref_logits = torch.from_numpy(z["logits"]).view(torch.float16).float()
    assert logits.shape == ref_logits.shape
    err = (logits.float() - ref_logits).abs().max().item()
    scale = ref_logits.abs().max().item()
    assert err <= LOGIT_TOL * scale, (err, scale)
    assert tokens == z["tokens"].tolist()
    assert int(z["swapped"][0]) == n_layer * (5 if kind == "llama" else 7)


def test_oracle_packer_restatement_matches_product_packer():
    for K, N, M, seed in ((256, 128, 4, 0), (1024, 256, 64, 9)):
        a = make_sparse_ref(K, N, M, seed)
        b = make_sparse(K, N, M, seed, "cpu")
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
