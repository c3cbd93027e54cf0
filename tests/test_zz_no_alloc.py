"""The allocation-free output-head entry point (nms_gemv_argmax_noalloc_f16).

It exists for callers that cannot allocate device memory per call -- a
serving runtime that has reserved the whole GPU for its own pools, or a C FFI
caller without a caching allocator -- and keeps its argmax scratch in a static
device array inside the library.  This test calls it through the C ABI and
checks it against the allocating entry point (nms_gemv_fused_f16 with the
dense argmax epilogue and caller-provided scratch) on two calls in a row, so
the second call also proves the shared scratch was left in a usable state.
Tolerance: the tests' GEMV bound (max-rel-error 2e-3 of the logits; the two
paths run the same kernel, so the logits are in fact identical) and the same
greedy token.  The file is named to be collected last.
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
    a.prologue = _lib.NMS_PRO_RESID_RMSNORM
    a.flags = _lib.NMS_FLAG_DENSE
    a.K = a.w = a.w_pad = head.shape[1]
    a.x, a.x2, a.norm_weight, a.eps = x.data_ptr(), x2.data_ptr(), norm.data_ptr(), 1e-5
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
            x.data_ptr(), x2.data_ptr(), norm.data_ptr(), ctypes.c_float(1e-5), head.data_ptr(), head.shape[0],
            head.shape[1], logits.data_ptr(), token.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
            "nms_gemv_argmax_noalloc_f16")
    torch.cuda.synchronize(dev)


def test_no_alloc_head_matches_allocating_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda:0")
    V, K = 128256, 4096
    g = torch.Generator(device=dev).manual_seed(1234)
    head = (torch.randn(V, K, generator=g, device=dev) * 0.02).to(torch.float16)
    norm = (1 + 0.1 * torch.randn(K, generator=g, device=dev)).to(torch.float16)
    for call in range(2):
        x = torch.randn(K, generator=g, device=dev).to(torch.float16)
        x2 = torch.randn(K, generator=g, device=dev).to(torch.float16)
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
        assert int(got_tok.item()) == int(torch.argmax(ref_logits).item()), call
    assert _lib.device_error() == 0
