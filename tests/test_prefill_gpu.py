"""Batched prefill (DecodeEngine.prefill: every N:M projection as one sparse
tensor-core GEMM over the prompt) against the reference's own decode path.

The reference fixtures (tests/golden) hold the reference decode path's
logits at every position.  The engine prefills all prompt tokens but the
last in one pass, then decodes teacher-forced on the fixture's tokens; the
logits at every position from the last prefilled one on must be within
LOGIT_TOL * max|logit| of the fixture's (the bar of the decode tests), which
also checks the K/V the prefill wrote, since every later step attends to
them.  The greedy token must equal the fixture's unless the fixture's
margin between the two tokens is within twice that step's logit error (an
fp16 near-tie that summation order decides).
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from spmv_decode_b200 import _lib
from spmv_decode_b200.engine import DecodeEngine
from spmv_decode_b200.generate import decode_one_token, generate
from test_decode_gpu import LOGIT_TOL, _f16, _model_from_golden

pytestmark = pytest.mark.gpu


def _check(got, ref, tok_got, tok_ref):
    got, ref = got.float().cpu(), ref.float()
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= LOGIT_TOL * scale, err / scale
    if tok_got != tok_ref:
        margin = (ref[tok_ref] - ref[tok_got]).item()
        assert margin <= 2 * err, (tok_got, tok_ref, margin, err)


@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_prefill_then_decode_matches_reference_fixture(cuda_device, kind):
    z = np.load(GOLDEN / f"decode_{kind}_tiny.npz")
    model, prompt_len, steps = _model_from_golden(z, kind, cuda_device)
    eng = DecodeEngine(model, 64, history_len=64)
    prompt = z["prompt"].tolist()
    toks_ref = z["tokens"].tolist()
    ref = _f16(z["logits"])
    P = len(prompt)
    inputs = prompt + toks_ref[:-1]
    last = eng.prefill(prompt[:-1])
    assert int(eng.pos.item()) == P - 1
    _check(last, ref[P - 2], int(torch.argmax(last)), int(torch.argmax(ref[P - 2].float())))
    for pos in range(P - 1, len(inputs)):
        tok, logits = decode_one_token(eng, inputs[pos], pos)
        _check(logits, ref[pos], tok, toks_ref[pos - (P - 1)])
    assert _lib.device_error() == 0
    eng.close()


def test_generate_with_batched_prefill(cuda_device):
    """Prefill of the whole prompt gives the reference's logits at the last
    prompt position; generate(batched_prefill=True) then returns the
    requested tokens, the first one the reference's (up to a near-tie)."""
    z = np.load(GOLDEN / "decode_llama_tiny.npz")
    model, prompt_len, steps = _model_from_golden(z, "llama", cuda_device)
    eng = DecodeEngine(model, 64, history_len=64)
    prompt = z["prompt"].tolist()
    toks_ref = z["tokens"].tolist()
    ref = _f16(z["logits"])
    P = len(prompt)
    last = eng.prefill(prompt)
    _check(last, ref[P - 1], int(torch.argmax(last)), toks_ref[0])
    toks = generate(eng, prompt, 8, batched_prefill=True)
    assert len(toks) == 8
    r = ref[P - 1].float()
    if toks[0] != toks_ref[0]:
        assert (r[toks_ref[0]] - r[toks[0]]).item() <= 2 * LOGIT_TOL * r.abs().max().item()
    with pytest.raises(ValueError):
        eng.prefill([])
    with pytest.raises(ValueError):
        eng.prefill([1] * 70)
    assert _lib.device_error() == 0
    eng.close()
