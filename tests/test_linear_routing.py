"""NmSparseLinear's multi-token routing (host logic, CPU): the reference
rule for T > 1 (src/spmv/nmsparse_linear.py:55-68) and the sparse_prefill()
switch the decode engine's batched prefill uses."""
import pytest
import torch


def test_multi_token_routing_keeps_the_reference_rule_on_cpu():
    """T > 1: dense F.linear when a dense weight is kept, RuntimeError when
    none is (src/spmv/nmsparse_linear.py:55-68); sparse_prefill() only
    reroutes CUDA input and restores its flag on exit."""
    import torch.nn.functional as F

    from spmv_decode_b200 import nmsparse_linear as NL

    dense = (torch.randn(128, 256) * 0.02).to(torch.float16)
    lin = NL.NmSparseLinear(128, 256, 32, 0, "cpu", dense_weight=dense)
    x = torch.randn(1, 3, 256).to(torch.float16)
    torch.testing.assert_close(lin(x), F.linear(x, dense))
    bare = NL.NmSparseLinear(128, 256, 32, 0, "cpu")
    with pytest.raises(RuntimeError, match="prefill requires dense weight"):
        bare(x)
    with NL.sparse_prefill():
        assert NL._SPARSE_PREFILL
        torch.testing.assert_close(lin(x), F.linear(x, dense))
    assert not NL._SPARSE_PREFILL
    with pytest.raises(KeyError):
        with NL.sparse_prefill():
            raise KeyError("x")
    assert not NL._SPARSE_PREFILL
