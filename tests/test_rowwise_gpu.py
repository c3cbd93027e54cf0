"""Per-row N:M GEMV (nms_gemv_rowwise_f16 through nmsparse::gemv) against the
oracle.  W fp16 [4096, 4096] ~ N(0, 0.02) seed 0, per-row
top-|w| 32:64, x ~ N(0, 1); tolerance max-rel-error <= 1e-2 (north star),
asserted <= 2e-3, against the fp32 product of the oracle's per-row layout."""
import numpy as np
import pytest
import torch

from oracle.nm_oracle import rowwise_gemv_fp32
from spmv_decode_b200 import nmsparse_op  # noqa: F401  (registers the op)
from spmv_decode_b200.nmsparse_linear import make_rowwise_topk

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _max_rel(y, ref):
    return float(np.abs(y.astype(np.float32) - ref).max() / np.abs(ref).max())


def _run(W, x, n, m, dev):
    md, mi = make_rowwise_topk(W.to(dev), n, m)
    w, h = md.shape
    y = torch.ops.nmsparse.gemv(x.to(dev), md, mi, w, h, n, m)
    torch.cuda.synchronize()
    ref = rowwise_gemv_fp32(x.cpu().numpy(), md.cpu().numpy(), mi.cpu().numpy(), n, m)
    return y.cpu().numpy().reshape(-1), ref


def test_config1_rowwise_gemv(cuda_device):
    torch.manual_seed(0)
    W = (torch.randn(4096, 4096) * 0.02).to(torch.float16)
    x = torch.randn(1, 4096).to(torch.float16)
    y, ref = _run(W, x, 32, 64, cuda_device)
    assert _max_rel(y, ref) <= TOL


@pytest.mark.parametrize("nm", [(2, 4), (4, 8), (8, 16), (16, 32), (64, 128), (128, 256)])
def test_rowwise_ratio_sweep(cuda_device, nm):
    g = torch.Generator().manual_seed(1)
    W = (torch.randn(4096, 4096, generator=g) * 0.02).to(torch.float16)
    x = torch.randn(1, 4096, generator=g).to(torch.float16)
    y, ref = _run(W, x, nm[0], nm[1], cuda_device)
    assert _max_rel(y, ref) <= TOL


@pytest.mark.parametrize("shape", [(6144, 4096), (28672, 4096), (4096, 14336), (128, 512)])
def test_rowwise_shapes(cuda_device, shape):
    h, K = shape
    g = torch.Generator(device=cuda_device).manual_seed(2)
    W = (torch.randn(h, K, generator=g, device=cuda_device) * 0.02).to(torch.float16)
    x = torch.randn(1, K, generator=g, device=cuda_device).to(torch.float16)
    y, ref = _run(W, x, 32, 64, cuda_device)
    assert _max_rel(y, ref) <= TOL


@pytest.mark.parametrize("M", [16, 64])
def test_rowwise_module_with_the_reference_packer(cuda_device, M):
    """NmSparseLinear(layout="rowwise") holds the reference packer's per-row
    values and offsets (NM_KERNEL=fp16_split layout, repeated offsets
    included) and decodes through nmsparse::gemv's per-row kernel."""
    from spmv_decode_b200.nmsparse_linear import NmSparseLinear

    K, N = 4096, 4096
    lin = NmSparseLinear(N, K, M, 0, cuda_device, layout="rowwise")
    x = torch.randn(1, 1, K, generator=torch.Generator().manual_seed(M)).to(torch.float16)
    y = lin(x.to(cuda_device))
    assert y.shape == (1, 1, N) and y.dtype == torch.float16
    ref = rowwise_gemv_fp32(x.numpy().reshape(-1), lin.mat_data.cpu().numpy(), lin.mat_index.cpu().numpy(),
                            M // 2, M)
    assert _max_rel(y.cpu().numpy().reshape(-1), ref) <= TOL


def test_engine_refuses_rowwise_layers(cuda_device):
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.model import ModelArgs, Transformer
    from spmv_decode_b200.nmsparse_linear import swap_to_nmsparse

    args = ModelArgs(block_size=64, vocab_size=256, n_layer=1, n_head=2, n_local_heads=1, dim=256,
                     intermediate_size=512)
    with torch.device(cuda_device):
        model = Transformer(args)
    model = model.half()
    swap_to_nmsparse(model, 32, cuda_device, layout="rowwise")
    with pytest.raises(NotImplementedError, match="per-row"):
        DecodeEngine(model, 32)
