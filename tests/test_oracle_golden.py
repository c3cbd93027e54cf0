"""Pin the oracle and the product packer to the reference's own outputs.

tests/golden/*.npz were produced by tests/golden/make_golden.py from the
reference code itself (the reference packer and the reference Triton kernels
under the Triton interpreter).  CPU only.
"""
import ctypes
import hashlib

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import nm_oracle as O
from spmv_decode_b200.nmsparse_linear import make_sparse, masked_dense


def _load(name):
    return np.load(GOLDEN / name)


def _cases(z, prefix):
    return sorted({k.split("_")[0] for k in z.files if k.startswith(prefix)})


def test_packer_bit_exact_small():
    """make_sparse == reference _make_sparse, byte for byte (shared-mask branch)."""
    z = _load("packer.npz")
    cases = _cases(z, "small")
    assert len(cases) == 7
    for c in cases:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        md, mi, w2, nnz2 = make_sparse(K, N, M, seed, "cpu")
        assert (w2, nnz2) == (w, nnz)
        assert md.dtype == torch.float16 and tuple(md.shape) == (w, N)
        assert mi.dtype == torch.uint8 and tuple(mi.shape) == (K // M, nnz)
        np.testing.assert_array_equal(md.view(torch.int16).numpy(), z[f"{c}_mat_data"])
        np.testing.assert_array_equal(mi.numpy(), z[f"{c}_mat_index"])


def test_packer_bit_exact_llama_shapes():
    """SHA-256 of the packed bytes at Llama shapes and the sweep's extreme ratios."""
    z = _load("packer.npz")
    cases = _cases(z, "big")
    assert len(cases) == 6
    for c in cases:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        md, mi, _, _ = make_sparse(K, N, M, seed, "cpu")
        np.testing.assert_array_equal(md[0, :16].view(torch.int16).numpy(), z[f"{c}_head_data"])
        np.testing.assert_array_equal(mi[:2].numpy(), z[f"{c}_head_index"])
        assert hashlib.sha256(md.view(torch.int16).numpy().tobytes()).digest() == z[f"{c}_sha_data"].tobytes()
        assert hashlib.sha256(mi.numpy().tobytes()).digest() == z[f"{c}_sha_index"].tobytes()


def test_first_values_match_survey_record():
    md, mi, w, nnz = make_sparse(4096, 4096, 64, 0, "cpu")
    assert (w, nnz) == (2048, 32)
    assert md[0, :4].tolist() == [-0.0175933837890625, -0.01800537109375, -0.00391387939453125,
                                  -0.006778717041015625]
    assert mi[0, :8].tolist() == [0, 2, 3, 4, 6, 8, 10, 11]


def test_oracle_matches_reference_kernel():
    """oracle gemv_fp32 == reference Triton kernels (generic and A100 variants)
    up to fp32 summation order, at every ratio from 2:4 to 128:256."""
    z = _load("gemv.npz")
    cases = _cases(z, "c")
    ratios = set()
    for c in cases:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        ratios.add((nnz, M))
        ref = O.gemv_fp32(z[f"{c}_vec"], z[f"{c}_mat_data"], z[f"{c}_mat_index"], K, M)
        scale = np.abs(ref).max()
        for variant in ("generic", "a100"):
            acc = z[f"{c}_acc_{variant}"].reshape(-1)
            assert np.abs(acc - ref).max() <= 1e-5 * scale, (c, variant)
        # The op's fp16 result is the rounded accumulator.
        op = O.as_f16(z[f"{c}_op_out"]).astype(np.float32)
        np.testing.assert_array_equal(op, z[f"{c}_acc_generic"].reshape(-1).astype(np.float16).astype(np.float32))
    assert {(2, 4), (4, 8), (8, 16), (16, 32), (32, 64), (64, 128), (128, 256)} <= ratios


def test_oracle_masked_dense_is_the_microbench_scatter():
    z = _load("gemv.npz")
    K, N, M, seed, w, nnz = (int(v) for v in z["c3_cfg"])
    dense = O.masked_dense(z["c3_mat_data"], z["c3_mat_index"], K, M)
    # exactly nnz non-zero columns per group, all rows share them
    nz_cols = np.nonzero(np.abs(dense.astype(np.float32)).sum(axis=0))[0]
    assert len(nz_cols) == w
    x = O.as_f16(z["c3_vec"]).reshape(-1).astype(np.float32)
    np.testing.assert_allclose(dense.astype(np.float32) @ x,
                               O.gemv_fp32(z["c3_vec"], z["c3_mat_data"], z["c3_mat_index"], K, M),
                               rtol=1e-5, atol=1e-5)
    # the product's torch restatement agrees bit for bit
    md = torch.from_numpy(z["c3_mat_data"]).view(torch.float16)
    mi = torch.from_numpy(z["c3_mat_index"])
    np.testing.assert_array_equal(masked_dense(md, mi, K, M).numpy(), dense)


def test_kernel_order_restatement():
    z = _load("gemv.npz")
    for c in ("c0", "c4"):
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        ko = O.gemv_kernel_order(z[f"{c}_vec"], z[f"{c}_mat_data"], z[f"{c}_mat_index"], M)
        ref = z[f"{c}_acc_generic"].reshape(-1)
        assert np.abs(ko - ref).max() <= 1e-5 * np.abs(ref).max()


def test_c_oracle_matches_reference_kernel(oracle_lib):
    z = _load("gemv.npz")
    for c in _cases(z, "c"):
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        vec = np.ascontiguousarray(z[f"{c}_vec"].reshape(-1).view(np.uint16))
        md = np.ascontiguousarray(z[f"{c}_mat_data"].view(np.uint16))
        mi = np.ascontiguousarray(z[f"{c}_mat_index"])
        out = np.zeros(N, dtype=np.float32)
        oracle_lib.nm_gemv_ref(vec.ctypes.data, md.ctypes.data, mi.ctypes.data, out.ctypes.data, K, w, N, nnz, M, 1)
        # gpp=1 with in-order partial sums is the generic kernel's order up
        # to the atomic-add order of its group programs.
        ref = z[f"{c}_acc_generic"].reshape(-1)
        assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max(), c


@pytest.mark.parametrize("n,m", [(2, 4), (16, 32), (32, 64), (128, 256)])
def test_rowwise_topk_packer_roundtrip(n, m):
    """Per-row top-|w|: unpack(pack(W)) == mask * W bit-exact,
    n kept per row and group, each kept |w| >= every dropped |w| of its group."""
    rng = np.random.default_rng(0)
    h, K = 64, 4 * m
    W = (rng.standard_normal((h, K)) * 0.02).astype(np.float16)
    vals, offs = O.rowwise_topk(W, n, m)
    assert vals.shape == (K // m * n, h) and offs.dtype == np.uint8
    dense = O.rowwise_masked_dense(vals, offs, K, n, m)
    mask = dense != 0
    np.testing.assert_array_equal(dense[mask], W[mask])
    A = np.abs(W.astype(np.float32)).reshape(h, K // m, m)
    kept = mask.reshape(h, K // m, m)
    assert (kept.sum(axis=2) == n).all()
    assert (np.where(kept, A, np.inf).min(axis=2) >= np.where(kept, -np.inf, A).max(axis=2)).all()
    x = rng.standard_normal(K).astype(np.float16)
    np.testing.assert_allclose(O.rowwise_gemv_fp32(x, vals, offs, n, m),
                               dense.astype(np.float32) @ x.astype(np.float32), rtol=1e-4, atol=1e-5)


def test_shared_mask_topk_packer():
    rng = np.random.default_rng(1)
    h, K, n, m = 32, 256, 16, 32
    W = (rng.standard_normal((h, K)) * 0.02).astype(np.float16)
    md, mi = O.shared_mask_topk(W, n, m)
    assert md.shape == (K // m * n, h) and mi.shape == (K // m, n)
    assert (np.diff(mi.astype(int), axis=1) > 0).all()
    dense = O.masked_dense(md, mi, K, m)
    cols = O.gather_columns(mi, m)
    np.testing.assert_array_equal(dense[:, cols], W[:, cols])


def test_gemm_oracle_is_the_gemv_oracle_row_by_row():
    """gemm_fp32 (multi-token oracle) equals gemv_fp32 on every token."""
    from oracle import nm_oracle as O2

    rng = np.random.default_rng(3)
    K, m, n, h, T = 512, 16, 8, 96, 5
    G = K // m
    mi = np.stack([np.sort(rng.permutation(m)[:n]) for _ in range(G)]).astype(np.uint8)
    md = (rng.standard_normal((G * n, h)) * 0.05).astype(np.float16)
    X = rng.standard_normal((T, K)).astype(np.float16)
    Y = O2.gemm_fp32(X, md, mi, K, m)
    assert Y.shape == (T, h) and Y.dtype == np.float32
    for t in range(T):
        np.testing.assert_allclose(Y[t], O2.gemv_fp32(X[t], md, mi, K, m), rtol=1e-5, atol=1e-6)
