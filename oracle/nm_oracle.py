"""ORACLE -- test infrastructure, not product code (see oracle/__init__.py).

numpy restatement of the reference's shared-mask N:M sparse GEMV:

* masked_dense  -- microbench_triton_torchmv.py:145-164: the dense [h, K]
  matrix with mat_data scattered to columns g*M + mat_index[g, i].
* gemv_fp32     -- microbench_triton_torchmv.py:383-386: torch.mv of that
  matrix and the vector, both in fp32 (the reference's correctness oracle).
* gemm_fp32     -- the same product for T tokens, row by row (the
  multi-token sparse layer the reference lacks, src/spmv/nmsparse_linear.py:55-68).
* gemv_kernel_order -- triton_spmv.py:81-108 loop order for one program
  (group by group, kept slot by kept slot, fp32 fused multiply-add); small
  cases only.
* metrics       -- microbench_triton_torchmv.py:401-423 plus the normwise
  max relative error used by the parity bar.
* Magnitude packers for dense weights: shared-mask
  top-n by column mass per group, and per-row top-|w| into the reference's
  per-row layout (values [w, h] + uint8 offsets [w, h],
  src/spmv/nmsparse_linear.py:27-29).  Ties go to the lower column index.

Pinned by tests/test_oracle_golden.py against tests/golden/gemv.npz, the
output of the reference Triton kernels run by the Triton interpreter.
"""
from __future__ import annotations

import numpy as np


def as_f16(a) -> np.ndarray:
    """int16 bit patterns (how fixtures store fp16) -> float16 view."""
    a = np.asarray(a)
    return a.view(np.float16) if a.dtype == np.int16 else a.astype(np.float16)


def gather_columns(mat_index: np.ndarray, m: int) -> np.ndarray:
    """Input column of every compressed position j (length w)."""
    G, n = mat_index.shape
    return (np.arange(G, dtype=np.int64)[:, None] * m + mat_index.astype(np.int64)).reshape(-1)


def masked_dense(mat_data: np.ndarray, mat_index: np.ndarray, K: int, m: int) -> np.ndarray:
    """[h, K] fp16 dense matrix of the kept values (reference layout input [w, h])."""
    mat_data = as_f16(mat_data)
    w, h = mat_data.shape
    cols = gather_columns(mat_index, m)
    assert cols.shape[0] == w
    dense = np.zeros((h, K), dtype=np.float16)
    dense[:, cols] = mat_data.T
    return dense


def gemv_fp32(x: np.ndarray, mat_data: np.ndarray, mat_index: np.ndarray, K: int, m: int) -> np.ndarray:
    """fp32 reference output [h]: masked dense fp32 matrix times fp32 vector."""
    x = as_f16(x).reshape(-1).astype(np.float32)
    assert x.shape[0] == K
    cols = gather_columns(mat_index, m)
    xc = x[cols]  # identical to the dense product: zero columns contribute nothing
    return as_f16(mat_data).astype(np.float32).T @ xc


def gemm_fp32(X: np.ndarray, mat_data: np.ndarray, mat_index: np.ndarray, K: int, m: int) -> np.ndarray:
    """fp32 reference output [T, h] for T tokens: gemv_fp32 of every row of X.

    The reference has no multi-token sparse product (its linear sends T > 1
    to a dense F.linear, src/spmv/nmsparse_linear.py:55-68), so each token's
    row is defined as its single-token product (microbench_triton_torchmv.py:383-386)."""
    X = as_f16(X).reshape(-1, K).astype(np.float32)
    cols = gather_columns(mat_index, m)
    return X[:, cols] @ as_f16(mat_data).astype(np.float32)


def gemv_kernel_order(x: np.ndarray, mat_data: np.ndarray, mat_index: np.ndarray, m: int) -> np.ndarray:
    """The reference kernel's accumulation order for a single program covering
    every group (fp32 fused multiply-add emulated in float64 then rounded)."""
    x = as_f16(x).reshape(-1).astype(np.float32)
    md = as_f16(mat_data).astype(np.float32)
    G, n = mat_index.shape
    h = md.shape[1]
    acc = np.zeros(h, dtype=np.float32)
    for g in range(G):
        for i in range(n):
            xi = x[g * m + int(mat_index[g, i])]
            acc = (md[g * n + i].astype(np.float64) * np.float64(xi) + acc.astype(np.float64)).astype(np.float32)
    return acc


def metrics(out: np.ndarray, ref: np.ndarray) -> dict:
    """max_abs, mean_abs, rmse, rel_l2 (microbench_triton_torchmv.py:401-423)
    and max_rel = max|out-ref| / max|ref| (the parity bar's max-rel-error)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(out - ref)
    return {
        "max_abs": float(diff.max()),
        "mean_abs": float(diff.mean()),
        "rmse": float(np.sqrt(np.mean(diff * diff))),
        "rel_l2": float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-12)),
        "max_rel": float(diff.max() / max(np.abs(ref).max(), 1e-12)),
    }


def shared_mask_topk(W: np.ndarray, n: int, m: int):
    """Shared-mask magnitude packer: per group of m input columns keep the n
    columns with the largest sum_r |W[r, c]| (ties -> lower column), sorted.
    Returns (mat_data [w, h] fp16, mat_index [K/m, n] uint8)."""
    W = as_f16(W)
    h, K = W.shape
    G = K // m
    mass = np.abs(W.astype(np.float32)).sum(axis=0).reshape(G, m)
    # Stable sort on -mass keeps the lower column first among equals.
    order = np.argsort(-mass, axis=1, kind="stable")[:, :n]
    idx = np.sort(order, axis=1).astype(np.uint8)
    cols = gather_columns(idx, m)
    return np.ascontiguousarray(W[:, cols].T), idx


def rowwise_topk(W: np.ndarray, n: int, m: int):
    """Per-row top-|w| packer: for every row and group of m
    columns keep the n largest |w| (ties -> lower column), ascending offsets.
    Returns (values [w, h] fp16, offsets [w, h] uint8) in the reference's
    per-row layout (src/spmv/nmsparse_linear.py:27-29)."""
    W = as_f16(W)
    h, K = W.shape
    G = K // m
    A = np.abs(W.astype(np.float32)).reshape(h, G, m)
    order = np.argsort(-A, axis=2, kind="stable")[:, :, :n]
    off = np.sort(order, axis=2)  # [h, G, n]
    vals = np.take_along_axis(W.reshape(h, G, m), off, axis=2)  # [h, G, n]
    values = np.ascontiguousarray(vals.reshape(h, G * n).T)
    offsets = np.ascontiguousarray(off.reshape(h, G * n).T.astype(np.uint8))
    return values, offsets


def rowwise_masked_dense(values: np.ndarray, offsets: np.ndarray, K: int, n: int, m: int) -> np.ndarray:
    """[h, K] dense matrix of a per-row layout (inverse of rowwise_topk)."""
    values = as_f16(values)
    w, h = values.shape
    j = np.arange(w)
    cols = (j // n)[:, None] * m + offsets.astype(np.int64)  # [w, h]
    dense = np.zeros((h, K), dtype=np.float16)
    dense[np.arange(h)[None, :].repeat(w, 0), cols] = values
    return dense


def rowwise_gemv_fp32(x: np.ndarray, values: np.ndarray, offsets: np.ndarray, n: int, m: int) -> np.ndarray:
    """fp32 output of the per-row layout: out[r] = sum_j v[j,r] x[(j//n)*m + off[j,r]]."""
    x = as_f16(x).reshape(-1).astype(np.float32)
    values = as_f16(values).astype(np.float32)
    w, h = values.shape
    cols = (np.arange(w) // n)[:, None] * m + offsets.astype(np.int64)
    return (values * x[cols]).sum(axis=0, dtype=np.float32)
