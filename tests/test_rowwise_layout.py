"""The reference's per-row layout as an NmSparseLinear layout (CPU).

The packer's per-row branch (NM_KERNEL=fp16 / fp16_split,
src/spmv/nmsparse_linear.py:27-29) is restated bit for bit: pinned against
tests/golden/packer_rowwise.npz, produced by the reference's own
_make_sparse.  The module keeps the reference layout (values [w, h],
offsets [w, h]); its dense equivalent, state-dict loading and multi-token
routing follow the reference.
"""
import hashlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN
from oracle import nm_oracle as O
from spmv_decode_b200.nmsparse_linear import NmSparseLinear, make_sparse, rowwise_masked_dense


def _sha(a: np.ndarray) -> bytes:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest()


def test_rowwise_packer_is_bit_exact_with_the_reference():
    z = np.load(GOLDEN / "packer_rowwise.npz")
    smalls = sorted({k.split("_")[0] for k in z.files if k.startswith("small")})
    assert smalls
    for c in smalls:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        md, mi, w2, nnz2 = make_sparse(K, N, M, seed, "cpu", layout="rowwise")
        assert (w2, nnz2) == (w, nnz) and tuple(mi.shape) == (w, N) and mi.dtype == torch.uint8
        assert np.array_equal(md.view(torch.int16).numpy(), z[f"{c}_mat_data"]), c
        assert np.array_equal(mi.numpy(), z[f"{c}_mat_index"]), c
    bigs = sorted({k.split("_")[0] for k in z.files if k.startswith("big")})
    for c in bigs:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        md, mi, _, _ = make_sparse(K, N, M, seed, "cpu", layout="rowwise")
        assert _sha(md.view(torch.int16).numpy()) == z[f"{c}_sha_data"].tobytes(), c
        assert _sha(mi.numpy()) == z[f"{c}_sha_index"].tobytes(), c


def test_rowwise_module_layout_and_dense_equivalent():
    K, N, M = 512, 128, 32
    lin = NmSparseLinear(N, K, M, 3, "cpu", layout="rowwise")
    assert lin.layout == "rowwise" and int(lin.mat_layout[0]) == 2
    assert tuple(lin.mat_data.shape) == (lin.w, N) and tuple(lin.mat_index.shape) == (lin.w, N)
    md, mi, _, _ = make_sparse(K, N, M, 3, "cpu", layout="rowwise")
    assert torch.equal(lin.reference_mat_data(), md) and torch.equal(lin.mat_index, mi)
    dense = lin.dense_masked_weight().float()
    x = torch.randn(K).to(torch.float16)
    ref = O.rowwise_gemv_fp32(x.numpy(), md.numpy(), mi.numpy(), M // 2, M)
    np.testing.assert_allclose((dense @ x.float()).numpy(), ref, rtol=2e-3, atol=2e-3)
    # Repeated offsets inside a group add both values at that input.
    assert torch.equal(rowwise_masked_dense(md, mi, K, M), lin.dense_masked_weight())


def test_rowwise_state_dict_and_multi_token_rule():
    K, N, M = 256, 128, 16
    a = NmSparseLinear(N, K, M, 1, "cpu", layout="rowwise")
    b = NmSparseLinear(N, K, M, 2, "cpu", layout="rowwise", init="empty")
    sd = {k: v for k, v in a.state_dict().items() if k != "mat_layout"}  # a reference state dict
    b.load_state_dict(sd)
    assert torch.equal(b.mat_data, a.mat_data) and torch.equal(b.mat_index, a.mat_index)
    x = torch.randn(1, 4, K).to(torch.float16)
    with pytest.raises(RuntimeError, match="prefill requires dense weight"):
        a(x)
    dense = (torch.randn(N, K) * 0.02).to(torch.float16)
    c = NmSparseLinear(N, K, M, 1, "cpu", dense_weight=dense, layout="rowwise")
    torch.testing.assert_close(c(x), F.linear(x, dense))
    with pytest.raises(ValueError):
        NmSparseLinear(N, K, M, 1, "cpu", layout="diagonal")


def test_tensor_parallel_sharding_refuses_rowwise_layers():
    from spmv_decode_b200.tp import shard_cols, shard_rows

    lin = NmSparseLinear(256, 512, 32, 0, "cpu", layout="rowwise")
    with pytest.raises(NotImplementedError, match="per-row"):
        shard_rows(lin, [(0, 128)])
    with pytest.raises(NotImplementedError, match="per-row"):
        shard_cols(lin, 0, 256)
    shared = NmSparseLinear(256, 512, 32, 0, "cpu", layout="shared")
    part = shard_rows(shared, [(0, 128)])
    assert part.layout == "shared" and part.h == 128
