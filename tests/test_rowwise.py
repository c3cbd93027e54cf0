"""Per-row N:M: the product's top-|w| packer against the
oracle's restatement, bit-exact, including ties (lower column wins) and the
round trip back to the masked dense matrix.  CPU only."""
import numpy as np
import pytest
import torch

from oracle.nm_oracle import rowwise_masked_dense, rowwise_topk
from spmv_decode_b200.nmsparse_linear import make_rowwise_topk


@pytest.mark.parametrize("nm", [(2, 4), (4, 8), (16, 32), (32, 64), (128, 256)])
def test_rowwise_packer_matches_oracle(nm):
    n, m = nm
    g = torch.Generator().manual_seed(3)
    W = (torch.randn(256, 512, generator=g) * 0.02).to(torch.float16)
    md, mi = make_rowwise_topk(W, n, m)
    ov, oo = rowwise_topk(W.numpy(), n, m)
    assert np.array_equal(md.numpy().view(np.uint16), ov.view(np.uint16))
    assert np.array_equal(mi.numpy(), oo)


def test_rowwise_packer_ties_go_to_lower_column():
    # Values from a tiny alphabet: many equal |w| inside a group.
    g = torch.Generator().manual_seed(4)
    W = (torch.randint(-2, 3, (128, 256), generator=g).float() * 0.5).to(torch.float16)
    md, mi = make_rowwise_topk(W, 16, 32)
    ov, oo = rowwise_topk(W.numpy(), 16, 32)
    assert np.array_equal(mi.numpy(), oo)
    assert np.array_equal(md.numpy().view(np.uint16), ov.view(np.uint16))


def test_rowwise_config1_round_trip():
    """4096 x 4096, 32:64, W ~ N(0, 0.02) seed 0: the kept values are exactly
    the 32 largest |w| of each row and group, and unpacking restores mask * W."""
    torch.manual_seed(0)
    W = (torch.randn(4096, 4096) * 0.02).to(torch.float16)
    md, mi = make_rowwise_topk(W, 32, 64)
    assert md.shape == (2048, 4096) and mi.shape == (2048, 4096)
    dense = rowwise_masked_dense(md.numpy(), mi.numpy(), 4096, 32, 64)
    Wn = W.numpy()
    kept = dense != 0
    assert np.array_equal(dense[kept], Wn[kept])
    # Every group keeps 32 columns whose |w| is >= every dropped |w| of the group.
    A = np.abs(Wn.astype(np.float32)).reshape(4096, 64, 64)
    mi3 = mi.numpy().T.reshape(4096, 64, 32).astype(np.int64)
    keep = np.zeros_like(A, dtype=bool)
    np.put_along_axis(keep, mi3, True, axis=2)
    assert keep.sum(axis=2).min() == 32
    lo_kept = np.where(keep, A, np.inf).min(axis=2)
    hi_drop = np.where(~keep, A, -np.inf).max(axis=2)
    assert (lo_kept >= hi_drop).all()

