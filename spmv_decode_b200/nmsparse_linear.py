"""NmSparseLinear and swap_to_nmsparse on the B200 packed layout.

Mirrors src/spmv/nmsparse_linear.py of the reference:

* ``make_sparse(K, N, M, seed, device)`` restates the reference packer
  ``_make_sparse`` (src/spmv/nmsparse_linear.py:14-33) in its shared-mask
  form (NM_KERNEL=triton_ptx): the same seeded CPU generator, the same draw
  order, so ``mat_data`` [w, N] and ``mat_index`` [K/M, M/2] are bit-exact
  with the reference's.
* ``NmSparseLinear(N, K, M, seed, device, dense_weight=None)`` has the
  reference constructor, attributes ``h, w, block_width, vec_width``,
  buffers ``mat_data`` and ``mat_index`` and forward rule (single token ->
  sparse GEMV, otherwise ``F.linear`` with the dense weight,
  :55-68).  Where the reference raises for want of a dense weight, a CUDA
  input runs the sparse layer on the tensor cores (``nmsparse::gemm_packed``).  The difference is storage: ``mat_data`` holds the packed layout
  [h, w_pad] (row-major transpose, 16-byte aligned rows) that the sm_100a
  kernel streams; ``reference_mat_data()`` returns the reference [w, h]
  layout, and reference state dicts load unchanged (they are repacked).
* ``swap_to_nmsparse(model, M, device, seed=0, block_devices=None)`` replaces
  the same linears in the same order with the same seeds (:71-144).

Environment variables ``NM_DECODE_ONLY`` and ``NM_WEIGHT_CPU`` keep the
reference meaning (:7-8).
"""
from __future__ import annotations

import contextlib
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import nmsparse_op  # noqa: F401  (registers torch.ops.nmsparse.*)
from .nmsparse_op import pack, packed_row_stride, unpack

DECODE_ONLY = os.environ.get("NM_DECODE_ONLY", "0") == "1"
WEIGHT_CPU = os.environ.get("NM_WEIGHT_CPU", "0") == "1" or DECODE_ONLY
# NM_KERNEL=fp16 / fp16_split select the reference's per-row layout
# (src/spmv/nmsparse_linear.py:9-11, 27-29); anything else accepted here
# (unset, triton_ptx) is the shared-mask layout.
DEFAULT_LAYOUT = "rowwise" if os.environ.get("NM_KERNEL", "") in ("fp16", "fp16_split") else "shared"

LAYOUT_PACKED = 1   # shared mask, values re-laid-out as packed [h, w_pad]
LAYOUT_ROWWISE = 2  # per-row offsets, values in the reference layout [w, h]

_SPARSE_PREFILL = False


@contextlib.contextmanager
def sparse_prefill(enabled: bool = True):
    """Inside the block, multi-token CUDA input to NmSparseLinear runs the
    sparse tensor-core GEMM even when a dense weight is kept -- the same
    weights single-token decode uses (the decode engine's batched prefill).
    Outside it the reference rule holds: dense ``F.linear`` when a dense
    weight is kept (src/spmv/nmsparse_linear.py:55-68)."""
    global _SPARSE_PREFILL
    old = _SPARSE_PREFILL
    _SPARSE_PREFILL = bool(enabled)
    try:
        yield
    finally:
        _SPARSE_PREFILL = old


def make_sparse(K: int, N: int, M: int, seed: int, device="cpu", *, layout: str = "shared"):
    """Synthetic N:M weights, bit-exact with the reference packer.

    ``layout="shared"`` (NM_KERNEL=triton_ptx): returns ``(mat_data [w, N]
    fp16, mat_index [K/M, M/2] uint8, w, nnz)`` -- one sorted random mask per
    group of M inputs shared by every output row (src/spmv/nmsparse_linear.py:14-33,
    branch :22-26).  ``layout="rowwise"`` (NM_KERNEL=fp16 / fp16_split): the
    same values and an offset in [0, M) drawn per value, ``mat_index [w, N]``
    uint8 (branch :27-29); offsets may repeat within a group, and the product
    then adds both values at that input.  50% sparsity (nnz = M/2) either way.
    """
    if layout not in ("shared", "rowwise"):
        raise ValueError(f"unknown layout={layout!r}")
    nnz = M // 2
    nb = K // M
    w = nb * nnz
    g = torch.Generator().manual_seed(seed)
    mat_data = (torch.randn(w, N, generator=g, dtype=torch.float32) / (K ** 0.5)).to(torch.float16)
    if layout == "rowwise":
        mat_index = torch.randint(0, M, (w, N), generator=g, dtype=torch.uint8)
    else:
        mat_index = torch.empty(nb, nnz, dtype=torch.uint8)
        for bank in range(nb):
            mat_index[bank] = torch.randperm(M, generator=g)[:nnz].sort().values.to(torch.uint8)
    if str(device) != "cpu":
        mat_data = mat_data.to(device)
        mat_index = mat_index.to(device)
    return mat_data, mat_index, w, nnz


def make_sparse_device(K: int, N: int, M: int, seed: int, device, std: float | None = None):
    """Synthetic shared-mask weights drawn directly on a CUDA device and
    packed there: same distribution as ``make_sparse`` (randn/sqrt(K), or
    N(0, std) when ``std`` is given; uniform random sorted in-group masks) but
    not the same numbers.  Used to build multi-GB benchmark models in seconds.

    Returns ``(packed [N, w_pad] fp16, mat_index [K/M, M/2] uint8, w, nnz)``.
    """
    nnz = M // 2
    nb = K // M
    w = nb * nnz
    gen = torch.Generator(device=device).manual_seed(seed)
    w_pad = packed_row_stride(w)
    packed = torch.zeros((N, w_pad), dtype=torch.float16, device=device)
    scale = std if std is not None else 1.0 / (K ** 0.5)
    # Draw in row blocks to bound the fp32 temporary.
    rows_per = max(1, (1 << 26) // max(w, 1))
    for r0 in range(0, N, rows_per):
        r1 = min(N, r0 + rows_per)
        blk = torch.randn((r1 - r0, w), generator=gen, dtype=torch.float32, device=device)
        packed[r0:r1, :w] = (blk * scale).to(torch.float16)
    keys = torch.rand((nb, M), generator=gen, device=device)
    mat_index = keys.argsort(dim=1)[:, :nnz].sort(dim=1).values.to(torch.uint8).contiguous()
    return packed, mat_index, w, nnz


def masked_dense(mat_data: torch.Tensor, mat_index: torch.Tensor, K: int, M: int) -> torch.Tensor:
    """Dense [h, K] weight with the kept values scattered back to their
    columns (the reference microbench's ``weight_sparse``,
    microbench_triton_torchmv.py:145-164).  Host/device agnostic."""
    w, h = mat_data.shape
    nb, nnz = mat_index.shape
    cols = (torch.arange(nb, device=mat_index.device).unsqueeze(1) * M + mat_index.long()).reshape(-1)
    dense = torch.zeros((h, K), dtype=mat_data.dtype, device=mat_data.device)
    dense[:, cols.to(mat_data.device)] = mat_data.t()
    return dense


def rowwise_masked_dense(mat_data: torch.Tensor, mat_index: torch.Tensor, K: int, M: int) -> torch.Tensor:
    """Dense [h, K] weight of the per-row layout (values [w, h], offsets
    [w, h]): value (j, r) added at column (j / N) * M + offset, N = w / (K / M).
    Repeated offsets accumulate, as the per-row product does."""
    w, h = mat_data.shape
    n = w // (K // M)
    base = (torch.arange(w, device=mat_index.device) // n * M).unsqueeze(1)
    cols = (base + mat_index.long()).t()  # [h, w]
    dense = torch.zeros((h, K), dtype=torch.float32, device=mat_data.device)
    dense.scatter_add_(1, cols.to(mat_data.device), mat_data.t().float())
    return dense.to(mat_data.dtype)


def make_rowwise_topk(weight: torch.Tensor, n: int, m: int):
    """Per-row top-|w| N:M packing of a dense [h, K] weight:
    for every row and group of m consecutive input columns keep the n largest
    |w| (ties go to the lower column), offsets ascending within the group.
    Returns (mat_data [w, h] fp16, mat_index [w, h] uint8) in the reference's
    per-row layout (src/spmv/nmsparse_linear.py:27-29), on weight's device."""
    h, K = weight.shape
    if K % m or n <= 0 or n > m or m > 256:
        raise ValueError(f"K={K} must be a multiple of M={m}, 0 < N <= M <= 256")
    G = K // m
    Wg = weight.to(torch.float16).reshape(h, G, m)
    # Stable descending sort keeps the lower column first among equal |w|.
    order = torch.sort(Wg.float().abs(), dim=2, descending=True, stable=True).indices[:, :, :n]
    off = torch.sort(order, dim=2).values
    vals = torch.gather(Wg, 2, off)
    mat_data = vals.reshape(h, G * n).t().contiguous()
    mat_index = off.reshape(h, G * n).t().contiguous().to(torch.uint8)
    return mat_data, mat_index


class NmSparseLinear(nn.Module):
    """50% N:M sparse linear (reference: src/spmv/nmsparse_linear.py:36-68).

    ``layout="shared"`` (default unless NM_KERNEL is fp16 / fp16_split): one
    mask per input group shared by all rows, values stored packed [h, w_pad]
    for the sm_100a GEMV and GEMM.  ``layout="rowwise"``: the reference's
    per-row layout, values [w, h] and offsets [w, h], decoded by the per-row
    kernel behind ``nmsparse::gemv``."""

    def __init__(self, N, K, M, seed, device, dense_weight=None, *, init: str = "reference",
                 layout: str | None = None):
        super().__init__()
        layout = DEFAULT_LAYOUT if layout is None else layout
        if layout not in ("shared", "rowwise"):
            raise ValueError(f"unknown layout={layout!r}")
        self.layout = layout
        assert K % M == 0 and N % 128 == 0, (K, N, M)
        self._weight_cpu = None
        self.weight = None
        if dense_weight is not None:
            if WEIGHT_CPU:
                self._weight_cpu = dense_weight.detach().cpu()
                del dense_weight
                if str(device) != "cpu" and torch.cuda.is_available():
                    torch.cuda.empty_cache()
            else:
                self.weight = dense_weight
        if layout == "rowwise":
            nnz = M // 2
            w = (K // M) * nnz
            if init == "reference":
                packed, mi, w, nnz = make_sparse(K, N, M, seed, device, layout="rowwise")
            elif init == "device":
                gen = torch.Generator(device=device).manual_seed(seed)
                packed = (torch.randn((w, N), generator=gen, device=device) / (K ** 0.5)).to(torch.float16)
                mi = torch.randint(0, M, (w, N), generator=gen, device=device, dtype=torch.uint8)
            elif init == "empty":
                packed = torch.zeros((w, N), dtype=torch.float16, device=device)
                mi = torch.zeros((w, N), dtype=torch.uint8, device=device)
            else:
                raise ValueError(f"unknown init={init!r}")
        elif init == "reference":
            md, mi, w, nnz = make_sparse(K, N, M, seed, device)
            packed = pack(md)
            del md
        elif init == "device":
            packed, mi, w, nnz = make_sparse_device(K, N, M, seed, device)
        elif init == "empty":
            nnz = M // 2
            w = (K // M) * nnz
            packed = torch.zeros((N, packed_row_stride(w)), dtype=torch.float16, device=device)
            mi = torch.zeros((K // M, nnz), dtype=torch.uint8, device=device)
        else:
            raise ValueError(f"unknown init={init!r}")
        self.register_buffer("mat_data", packed)
        self.register_buffer("mat_index", mi)
        code = LAYOUT_ROWWISE if layout == "rowwise" else LAYOUT_PACKED
        self.register_buffer("mat_layout", torch.tensor([code], dtype=torch.uint8, device=packed.device))
        self.h, self.w, self.block_width, self.vec_width = N, w, nnz, M
        self.in_features, self.out_features = K, N

    @property
    def w_pad(self) -> int:
        """Row stride of the packed values (shared layout); w for per-row."""
        return self.w if self.layout == "rowwise" else int(self.mat_data.shape[-1])

    def reference_mat_data(self) -> torch.Tensor:
        """The kept values in the reference layout [w, h] (bit-exact)."""
        return self.mat_data if self.layout == "rowwise" else unpack(self.mat_data, self.w)

    def dense_masked_weight(self) -> torch.Tensor:
        """[h, K] dense weight holding the kept values (zeros elsewhere)."""
        if self.layout == "rowwise":
            return rowwise_masked_dense(self.mat_data, self.mat_index, self.in_features, self.vec_width)
        return masked_dense(self.reference_mat_data(), self.mat_index, self.in_features, self.vec_width)

    def _prefill_weight(self, device):
        if self.weight is not None:
            return self.weight
        if self._weight_cpu is None:
            raise RuntimeError("prefill requires dense weight")
        return self._weight_cpu.to(device)

    def forward(self, x):
        if x.shape[-2] == 1:
            if self.layout == "rowwise":
                return torch.ops.nmsparse.gemv(
                    x, self.mat_data, self.mat_index,
                    self.w, self.h, self.block_width, self.vec_width,
                )
            return torch.ops.nmsparse.gemv_packed(
                x, self.mat_data, self.mat_index,
                self.w, self.h, self.block_width, self.vec_width,
            )
        if self.layout == "shared" and x.is_cuda and (
                _SPARSE_PREFILL or (self.weight is None and self._weight_cpu is None)):
            # No dense weight kept (the reference raises here, :57-61), or
            # inside sparse_prefill(): the sparse layer on the tensor cores.
            return torch.ops.nmsparse.gemm_packed(
                x, self.mat_data, self.mat_index,
                self.w, self.h, self.block_width, self.vec_width,
            )
        return F.linear(x, self._prefill_weight(x.device))

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        # A reference state dict has mat_data in [w, h] and no layout marker.
        key_d, key_l = prefix + "mat_data", prefix + "mat_layout"
        if self.layout == "rowwise":
            if key_d in state_dict and key_l not in state_dict:
                state_dict[key_l] = torch.tensor([LAYOUT_ROWWISE], dtype=torch.uint8)
        elif key_d in state_dict and key_l not in state_dict:
            md = state_dict[key_d]
            if tuple(md.shape) == (self.w, self.h):
                state_dict[key_d] = pack(md.to(torch.float16), self.w_pad)
                state_dict[key_l] = torch.tensor([LAYOUT_PACKED], dtype=torch.uint8)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    def extra_repr(self) -> str:
        return (f"in={self.in_features}, out={self.h}, {self.block_width}:{self.vec_width}, "
                f"w={self.w}, w_pad={self.w_pad}, layout={self.layout}")


# Block layouts swap_to_nmsparse knows (reference :83-91): gpt-fast fused
# attention (wqkv, wo) and MLP (w1, w3, w2); HF decoder blocks
# (q/k/v/o_proj, gate/up/down_proj).
_ATTENTION_LAYOUTS = (
    ("attention", ("wqkv", "wo")),
    ("self_attn", ("q_proj", "k_proj", "v_proj", "o_proj")),
)

_MLP_LAYOUTS = (
    ("feed_forward", ("w1", "w3", "w2")),
    ("mlp", ("gate_proj", "up_proj", "down_proj")),
)


def _resolve_layout(blk, layouts, kind):
    for submodule_attr, linear_names in layouts:
        submodule = getattr(blk, submodule_attr, None)
        if submodule is not None:
            return submodule, linear_names
    known = ", ".join(f".{attr}" for attr, _ in layouts)
    raise AttributeError(
        f"decoder block {type(blk).__name__} has none of the known "
        f"{kind} sub-modules ({known}); swap_to_nmsparse does not "
        f"recognize this block's layout."
    )


def _swap_linears(submodule, linear_names, M, device, seed, cnt, init, keep_dense, layout):
    for name in linear_names:
        old = getattr(submodule, name)
        if isinstance(old, NmSparseLinear):
            N, K = old.h, old.in_features
        else:
            N, K = old.weight.shape
        keep = (not DECODE_ONLY) if keep_dense is None else keep_dense
        dense_weight = old.weight if (keep and not isinstance(old, NmSparseLinear)) else None
        del old
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        setattr(submodule, name, NmSparseLinear(N, K, M, seed + cnt, device, dense_weight=dense_weight, init=init,
                                                layout=layout))
        cnt += 1
    return cnt


def swap_to_nmsparse(model, M, device, seed=0, block_devices=None, *, init: str = "reference",
                     keep_dense: bool | None = None, layout: str | None = None):
    """Replace every decoder block's attention and MLP linears with
    NmSparseLinear (reference: src/spmv/nmsparse_linear.py:124-144).

    Linear number ``cnt`` (in block order, attention then MLP, names in layout
    order) gets seed ``seed + cnt``.  ``block_devices`` optionally gives one
    device per block.  Returns the number of linears swapped.
    ``init="device"`` draws the weights on the GPU instead (same
    distribution, different numbers, much faster for multi-GB models).
    ``keep_dense`` overrides NM_DECODE_ONLY for keeping the dense weight (used
    by prefill with more than one token, :55-68).  ``layout`` ("shared" or
    "rowwise") overrides the NM_KERNEL default of NmSparseLinear.
    """
    cnt = 0
    for i, blk in enumerate(model.layers):
        blk_device = device
        if block_devices is not None:
            d = block_devices[i]
            blk_device = d if isinstance(d, str) else f"cuda:{d}"
        attn, attn_names = _resolve_layout(blk, _ATTENTION_LAYOUTS, "attention")
        cnt = _swap_linears(attn, attn_names, M, blk_device, seed, cnt, init, keep_dense, layout)
        mlp, mlp_names = _resolve_layout(blk, _MLP_LAYOUTS, "feed-forward")
        cnt = _swap_linears(mlp, mlp_names, M, blk_device, seed, cnt, init, keep_dense, layout)
    return cnt
