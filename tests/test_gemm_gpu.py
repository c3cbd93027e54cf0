"""GPU parity of the prefill / batch > 1 sparse GEMM (``nmsparse::gemm_packed``,
C-ABI nms_gemm_packed_f16) against the oracle.

Every token's row is the single-token N:M product (oracle gemm_fp32 = the
fp32 dense product of the masked weights, row by row).  Tolerance: the
north-star GEMV bar, max-rel-error <= 1e-2 with max-rel-error =
max |y - ref| / max |ref| over the whole [T, h] output, plus the tighter
2e-3 that fp32 accumulation with an fp16 result meets, to catch regressions
(5e-3 for a bf16 result: its 8-bit significand alone rounds by up to
2^-8 of max|ref|).
Inputs in bf16 or fp32 are converted to fp16 first, as the reference op
converts its input (src/spmv/nmsparse_op.py:88-90); the result comes back
in the input's dtype.
"""
import numpy as np
import pytest
import torch

from oracle import nm_oracle as O
from spmv_decode_b200 import _lib
from spmv_decode_b200.nmsparse_linear import NmSparseLinear, make_sparse, make_sparse_device
from spmv_decode_b200.nmsparse_op import pack, unpack

pytestmark = pytest.mark.gpu

TOL_MAX_REL = 1e-2
TOL_TIGHT = 2e-3


def _oracle(x: torch.Tensor, packed: torch.Tensor, mi: torch.Tensor, w: int, K: int, M: int) -> np.ndarray:
    md = unpack(packed, w).cpu().view(torch.int16).numpy()
    xh = x.reshape(-1, K).to(torch.float16).cpu().view(torch.int16).numpy()
    return O.gemm_fp32(xh, md, mi.cpu().numpy(), K, M)


TOL_TIGHT_BF16 = 5e-3


def _check(y: torch.Tensor, ref: np.ndarray):
    yy = y.float().reshape(ref.shape).cpu().numpy()
    assert np.isfinite(yy).all()
    m = O.metrics(yy, ref)
    assert m["max_rel"] <= TOL_MAX_REL, m
    assert m["max_rel"] <= (TOL_TIGHT_BF16 if y.dtype == torch.bfloat16 else TOL_TIGHT), m
    return m


def _device_error_clear():
    import ctypes

    code = ctypes.c_int32(0)
    _lib.check(_lib.lib().nms_device_error(ctypes.byref(code), 1), "nms_device_error")
    return code.value


def _layer(h, K, M, seed, device):
    lin = NmSparseLinear(h, K, M, seed, device, init="device")
    return lin


@pytest.mark.parametrize("T", [2, 5, 16, 17, 64, 128, 200, 256, 300, 512])
def test_reference_packer_4096(cuda_device, T):
    """Config-1 shape with the reference packer's values, every token count
    class: below one 16-token MMA, ragged, one tile, several token tiles."""
    K = h = 4096
    M = 64
    md, mi, w, nnz = make_sparse(K, h, M, 0, "cpu")
    packed = pack(md).to(cuda_device)
    mi = mi.to(cuda_device)
    g = torch.Generator(device="cpu").manual_seed(T)
    x = torch.randn(T, K, generator=g).to(torch.float16).to(cuda_device)
    y = torch.ops.nmsparse.gemm_packed(x, packed, mi, w, h, nnz, M)
    assert y.shape == (T, h) and y.dtype == torch.float16
    _check(y, _oracle(x, packed, mi, w, K, M))
    assert _device_error_clear() == 0


@pytest.mark.parametrize("n,m", [(2, 4), (4, 8), (8, 16), (16, 32), (32, 64), (64, 128), (128, 256)])
def test_ratio_sweep(cuda_device, n, m):
    K, h, T = 4096, 4096, 96
    lin = _layer(h, K, m, 1, cuda_device)
    assert lin.block_width == n
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    y = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, n, m)
    _check(y, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, m))


@pytest.mark.parametrize("h,K", [(6144, 4096), (28672, 4096), (4096, 14336)])
@pytest.mark.parametrize("T", [128, 512])
def test_llama_shapes(cuda_device, h, K, T):
    lin = _layer(h, K, 64, 2, cuda_device)
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    y = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, 64)
    _check(y, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, 64))


@pytest.mark.parametrize("h", [1, 8, 200, 129, 1000])
def test_ragged_rows(cuda_device, h):
    """Any h >= 1 on the packed layout: partial row tiles, and h % 8 != 0
    (element-wise output stores)."""
    K, M, T = 1024, 32, 40
    g = torch.Generator(device="cpu").manual_seed(h)
    G, n = K // M, M // 2
    mi = torch.stack([torch.randperm(M, generator=g)[:n].sort().values for _ in range(G)]).to(torch.uint8)
    md = (torch.randn(G * n, h, generator=g) * 0.05).to(torch.float16)
    packed = pack(md).to(cuda_device)
    mi = mi.to(cuda_device)
    x = torch.randn(T, K, generator=g).to(torch.float16).to(cuda_device)
    y = torch.ops.nmsparse.gemm_packed(x, packed, mi, G * n, h, n, M)
    _check(y, _oracle(x, packed, mi, G * n, K, M))


def test_w_not_multiple_of_64(cuda_device):
    """w = 800 (K = 1600 at 32:64): the last 64-column stage is half padding."""
    K, h, M, T = 1600, 256, 64, 33
    lin = _layer(h, K, M, 3, cuda_device)
    assert lin.w == 800 and lin.w_pad == 832
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    y = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    _check(y, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_input_dtypes(cuda_device, dtype):
    K, h, M, T = 4096, 1024, 64, 48
    lin = _layer(h, K, M, 4, cuda_device)
    x = torch.randn(3, T // 3, K, device=cuda_device).to(dtype)
    y = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    assert y.shape == (3, T // 3, h) and y.dtype == dtype
    _check(y, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M))


def test_split_k_is_deterministic(cuda_device):
    """Few tiles -> split-K with the fixed-order reduction: repeated launches
    give bit-identical results."""
    K, h, M, T = 14336, 4096, 64, 16
    lin = _layer(h, K, M, 5, cuda_device)
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    ys = [torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M) for _ in range(5)]
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    _check(ys[0], _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M))


def test_rows_agree_with_the_gemv(cuda_device):
    """Each token's row of the GEMM and the single-token GEMV are both within
    the tight bound of the oracle, hence within 2x of each other."""
    K, h, M, T = 4096, 6144, 64, 8
    lin = _layer(h, K, M, 6, cuda_device)
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    y = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    ref = _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M)
    for t in range(T):
        yv = torch.ops.nmsparse.gemv_packed(x[t].view(1, 1, K), lin.mat_data, lin.mat_index, lin.w, h, 32, M)
        _check(yv.reshape(1, h), ref[t:t + 1])
        d = (y[t].float() - yv.reshape(-1).float()).abs().max().item()
        assert d <= 2 * TOL_TIGHT * float(np.abs(ref[t]).max())


def test_linear_forward_uses_the_sparse_gemm_without_dense_weight(cuda_device):
    K, h, M = 2048, 1024, 64
    lin = NmSparseLinear(h, K, M, 7, cuda_device)
    x = torch.randn(2, 24, K, device=cuda_device).to(torch.float16)
    y = lin(x)
    assert y.shape == (2, 24, h)
    _check(y, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M))
    # With a dense weight kept, the reference rule (dense F.linear) stands.
    dense = torch.randn(h, K, device=cuda_device).to(torch.float16) * 0.02
    lin2 = NmSparseLinear(h, K, M, 7, cuda_device, dense_weight=dense)
    torch.testing.assert_close(lin2(x), torch.nn.functional.linear(x, dense))


def test_cuda_graph_capture(cuda_device):
    K, h, M, T = 4096, 4096, 64, 64
    lin = _layer(h, K, M, 8, cuda_device)
    x = torch.randn(T, K, device=cuda_device).to(torch.float16)
    eager = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = torch.ops.nmsparse.gemm_packed(x, lin.mat_data, lin.mat_index, lin.w, h, 32, M)
    x.copy_(torch.randn(T, K, device=cuda_device).to(torch.float16))
    graph.replay()
    torch.cuda.synchronize()
    _check(out, _oracle(x, lin.mat_data, lin.mat_index, lin.w, K, M))
    assert not torch.equal(out, eager)
    del graph
    assert _device_error_clear() == 0
