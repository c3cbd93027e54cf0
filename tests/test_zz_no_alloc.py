"""The allocation-free output-head entry point (nms_gemv_argmax_noalloc_f16).

It exists for callers that cannot allocate device memory per call -- a
serving runtime that has reserved the whole GPU for its own pools, or a C FFI
caller without a caching allocator -- and keeps its argmax scratch in a static
device array inside the library.  This test calls it through the C ABI and
checks it against the allocating entry point (nms_gemv_fused_f16 with the
dense argmax epilogue and caller-provided scratch) on two calls in a row, so
the second call also proves the shared scratch was left in a usable state.
Every prologue variant the header documents runs (residual add + RMSNorm,
RMSNorm without an addend, plain).  Tolerance: the tests' GEMV bound
(max-rel-error 2e-3 of the logits) against the allocating entry point (the
same kernel, so in fact identical) and against a plain PyTorch fp32
restatement at 128256 x 4096, and the same greedy token (the fp32 argmax up
to an fp16 near-tie).  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from spmv_decode_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _allocating_reference(x, x2, norm, head, logits, token):
    dev = x.device
    cap = 2048
    amax_val = torch.empty(cap, device=dev, dtype=torch.float32)
    amax_idx = torch.empty(cap, device=dev, dtype=torch.int32)
    counter = torch.zeros(1, device=dev, dtype=torch.int32)
    a = _lib.NmsGemvFusedArgs()
    a.seg[0].packed = head.data_ptr()
    a.seg[0].rows = head.shape[0]
    a.nseg = 1
    a.epilogue = _lib.NMS_EPI_ARGMAX
    a.prologue = _lib.NMS_PRO_RESID_RMSNORM if norm is not None else _lib.NMS_PRO_PLAIN
    a.flags = _lib.NMS_FLAG_DENSE
    a.K = a.w = a.w_pad = head.shape[1]
    a.x, a.x2 = x.data_ptr(), _lib.ptr(x2) if norm is not None else None
    a.norm_weight, a.eps = _lib.ptr(norm), 1e-5
    a.out = logits.data_ptr()
    a.amax_val, a.amax_idx = amax_val.data_ptr(), amax_idx.data_ptr()
    a.amax_counter, a.token_out, a.amax_capacity = counter.data_ptr(), token.data_ptr(), cap
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().nms_gemv_fused_f16(ctypes.byref(a), torch.cuda.current_stream(dev).cuda_stream))
    torch.cuda.synchronize(dev)


def _no_alloc(x, x2, norm, head, logits, token):
    dev = x.device
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().nms_gemv_argmax_noalloc_f16(
            x.data_ptr(), _lib.ptr(x2), _lib.ptr(norm), ctypes.c_float(1e-5), head.data_ptr(), head.shape[0],
            head.shape[1], logits.data_ptr(), token.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
            "nms_gemv_argmax_noalloc_f16")
    torch.cuda.synchronize(dev)


def _fp32_logits(x, x2, norm, head):
    """Plain PyTorch fp32 restatement: x (+ x2, rounded to fp16 like the
    reference's residual add), the reference RMSNorm roundings (fp32 norm,
    fp16 result, fp16 product with the weight), then head @ x in fp32."""
    xin = x
    if norm is not None:
        if x2 is not None:
            xin = (x.float() + x2.float()).to(torch.float16)
        xf = xin.float()
        xn = (xf * torch.rsqrt(torch.mean(xf * xf) + 1e-5)).to(torch.float16)
        xin = (xn.float() * norm.float()).to(torch.float16)
    return head.float() @ xin.float()


# Prologue variants the header documents: residual add + RMSNorm, RMSNorm
# without an addend (x2 = NULL), and the plain prologue (norm_weight = NULL).
VARIANTS = {"norm+x2": (True, True), "norm": (True, False), "plain": (False, False)}


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_no_alloc_head_matches_allocating_entry_point(variant):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    use_norm, use_x2 = VARIANTS[variant]
    dev = torch.device("cuda:0")
    V, K = 128256, 4096
    g = torch.Generator(device=dev).manual_seed(1234)
    head = (torch.randn(V, K, generator=g, device=dev) * 0.02).to(torch.float16)
    norm = (1 + 0.1 * torch.randn(K, generator=g, device=dev)).to(torch.float16) if use_norm else None
    for call in range(2):
        x = torch.randn(K, generator=g, device=dev).to(torch.float16)
        x2 = torch.randn(K, generator=g, device=dev).to(torch.float16) if use_x2 else None
        ref_logits = torch.empty(V, device=dev, dtype=torch.float16)
        ref_tok = torch.full((1,), -1, device=dev, dtype=torch.int64)
        _allocating_reference(x, x2, norm, head, ref_logits, ref_tok)
        got_logits = torch.full((V,), float("nan"), device=dev, dtype=torch.float16)
        got_tok = torch.full((1,), -1, device=dev, dtype=torch.int64)
        _no_alloc(x, x2, norm, head, got_logits, got_tok)
        diff = (got_logits.float() - ref_logits.float()).abs().max().item()
        scale = ref_logits.float().abs().max().item()
        assert diff <= TOL * scale, (call, diff, scale)
        assert int(got_tok.item()) == int(ref_tok.item()), call
        assert int(got_tok.item()) == int(torch.argmax(got_logits).item()), call
        # Against the fp32 restatement: logits within the tests' GEMV bound,
        # and the greedy token is the fp32 argmax unless the two are an fp16
        # near-tie (margin within the measured logit error).
        f32 = _fp32_logits(x, x2, norm, head)
        err = (got_logits.float() - f32).abs().max().item()
        fscale = f32.abs().max().item()
        assert err <= TOL * fscale, (call, err, fscale)
        t = int(got_tok.item())
        best = int(torch.argmax(f32).item())
        assert t == best or (f32[best] - f32[t]).item() <= 2 * err, (call, t, best)
    assert _lib.device_error() == 0
