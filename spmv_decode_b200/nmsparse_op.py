"""The ``nmsparse::gemv`` operator, backed by libnmsparse_b200 (sm_100a CUDA).

Drop-in for the reference operator boundary (src/spmv/nmsparse_op.py:77-123):
same op name, same signature, same fake kernel, same argument meaning and
the same exception types for the same conditions.  The reference selected a
backend from ``NM_KERNEL``; here there is exactly one backend and no
fallback.  ``NM_KERNEL`` unset or ``triton_ptx`` selects the shared-mask
layout, ``fp16`` or ``fp16_split`` the per-row layout (values [w, h], offsets
[w, h], served by the per-row kernel: the reference names CUDA kernels for it
that it does not ship); anything else -- ``guarded``, a CUDA-guard build for
tensor parallelism, or a typo -- raises ``ValueError`` like the reference's
allow-list (src/spmv/nmsparse_op.py:20-22).

Also registers ``nmsparse::gemv_packed`` for the re-laid-out weights that
``NmSparseLinear`` stores (packed [h, w_pad] rows, see include/nmsparse_b200.h),
and ``nmsparse::gemm_packed``, the same product for any number of tokens
(prefill / batch > 1) on the tensor cores.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_kernel = os.environ.get("NM_KERNEL", "")
if _kernel not in ("", "triton_ptx", "fp16", "fp16_split"):
    raise ValueError(
        f"Unknown NM_KERNEL={_kernel!r}; this build has one CUDA backend (shared-mask layout for "
        "NM_KERNEL unset / triton_ptx, per-row layout for fp16 / fp16_split) and refuses silent fallback"
    )
_mode = "b200_cuda"


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _validate_forward(vec: torch.Tensor, mat_data: torch.Tensor, mat_index: torch.Tensor,
                      w: int, h: int, block_width: int, vec_width: int, vec_num: int) -> None:
    """Host checks of the reference wrapper (triton_spmv.py:245-283), same
    exception types, plus the K == (w/N)*M consistency check that keeps the
    gather inside the vector."""
    if not vec.is_cuda or not mat_data.is_cuda or not mat_index.is_cuda:
        raise ValueError("vec, mat_data, and mat_index must be CUDA tensors")
    if vec.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported vec dtype: {vec.dtype}")
    if mat_data.dtype != vec.dtype:
        raise TypeError("vec and mat_data must have same dtype")
    if mat_index.dtype != torch.uint8:
        raise TypeError("mat_index must be uint8")
    if vec.ndim != 2 or vec.shape[0] != 1:
        raise ValueError(f"vec must have shape [1, {vec_num}]")
    if vec.shape[1] != vec_num:
        raise ValueError(f"vec.shape[1]={vec.shape[1]} != vecNum={vec_num}")
    if h % 128 != 0:
        raise ValueError("h must be divisible by 128")
    if block_width <= 0 or w % block_width != 0:
        raise ValueError(f"w={w} must be divisible by N={block_width}")
    num_groups = w // block_width
    if tuple(mat_data.shape) != (w, h):
        raise ValueError(f"mat_data must have shape {(w, h)}, got {tuple(mat_data.shape)}")
    # Shared mask [G, N]; or the per-row layout [w, h] (one offset per kept
    # value, src/spmv/nmsparse_linear.py:27-29).
    if tuple(mat_index.shape) not in ((num_groups, block_width), (w, h)):
        raise ValueError(
            f"mat_index must have shape {(num_groups, block_width)} (shared mask) or {(w, h)} (per-row), "
            f"got {tuple(mat_index.shape)}"
        )
    if not mat_data.is_contiguous():
        raise ValueError("mat_data must be contiguous")
    if not mat_index.is_contiguous():
        raise ValueError("mat_index must be contiguous")
    if not vec.is_contiguous():
        raise ValueError("vec must be contiguous")
    if num_groups * vec_width != vec_num:
        raise ValueError(f"vecNum={vec_num} != (w/N)*M = {num_groups * vec_width}")
    if mat_data.device != vec.device or mat_index.device != vec.device:
        raise ValueError("vec, mat_data and mat_index must be on the same device")


def nmsparse_spmv_forward(vec: torch.Tensor, mat_data: torch.Tensor, mat_index: torch.Tensor,
                          w: int, h: int, block_width: int, vec_width: int) -> torch.Tensor:
    """[1, K] fp16 x reference-layout weights -> [1, h] fp16 (the role of
    nmsparse_spmv_forward_triton_ptx, triton_spmv.py:229-318)."""
    K = vec.shape[-1]
    _validate_forward(vec, mat_data, mat_index, w, h, block_width, vec_width, K)
    if vec.dtype != torch.float16:
        raise TypeError("the sm_100a kernel computes fp16 x fp16 -> fp32; cast inputs to float16")
    out = torch.empty((1, h), dtype=torch.float16, device=vec.device)
    rowwise = tuple(mat_index.shape) == (w, h) and (w, h) != (w // block_width, block_width)
    fn = "nms_gemv_rowwise_f16" if rowwise else "nms_gemv_f16"
    with torch.cuda.device(vec.device):
        _lib.check(
            getattr(_lib.lib(), fn)(
                vec.data_ptr(), mat_data.data_ptr(), mat_index.data_ptr(), out.data_ptr(),
                int(K), int(w), int(h), int(block_width), int(vec_width), _stream_ptr(vec.device),
            ),
            fn,
        )
    return out


@torch.library.custom_op("nmsparse::gemv", mutates_args=())
def gemv(x: torch.Tensor, mat_data: torch.Tensor, mat_index: torch.Tensor,
         w: int, h: int, block_width: int, vec_width: int) -> torch.Tensor:
    """N:M GEMV on the reference layout (src/spmv/nmsparse_op.py:77-96):
    shared mask (mat_index [w/N, N]) or per-row mask (mat_index [w, h])."""
    K = x.shape[-1]
    x2d = x.reshape(-1, K).contiguous()
    if x2d.shape[0] != 1:
        raise RuntimeError(
            f"nmsparse gemv only supports decode (rows==1), got {tuple(x2d.shape)}"
        )
    xh = x2d if x2d.dtype == torch.float16 else x2d.to(torch.float16)
    md = mat_data if mat_data.dtype == torch.float16 else mat_data.to(torch.float16)
    out = nmsparse_spmv_forward(xh, md, mat_index, int(w), int(h), int(block_width), int(vec_width))
    out = out.to(dtype=x.dtype)
    return out.reshape(*x.shape[:-1], int(h))


@gemv.register_fake
def _(x, mat_data, mat_index, w, h, block_width, vec_width):
    return x.new_empty((*x.shape[:-1], int(h)))


@torch.library.custom_op("nmsparse::gemv_packed", mutates_args=())
def gemv_packed(x: torch.Tensor, mat_packed: torch.Tensor, mat_index: torch.Tensor,
                w: int, h: int, block_width: int, vec_width: int) -> torch.Tensor:
    """Shared-mask N:M GEMV on the packed layout [h, w_pad] (NmSparseLinear's
    storage).  Same arithmetic and contract as ``nmsparse::gemv``."""
    K = x.shape[-1]
    x2d = x.reshape(-1, K).contiguous()
    if x2d.shape[0] != 1:
        raise RuntimeError(
            f"nmsparse gemv only supports decode (rows==1), got {tuple(x2d.shape)}"
        )
    if not x.is_cuda or not mat_packed.is_cuda or not mat_index.is_cuda:
        raise ValueError("x, mat_packed, and mat_index must be CUDA tensors")
    if mat_index.dtype != torch.uint8:
        raise TypeError("mat_index must be uint8")
    xh = x2d if x2d.dtype == torch.float16 else x2d.to(torch.float16)
    if mat_packed.dtype != torch.float16:
        raise TypeError("mat_packed must be float16")
    w_pad = mat_packed.shape[-1]
    if mat_packed.ndim != 2 or mat_packed.shape[0] != h or not mat_packed.is_contiguous():
        raise ValueError(f"mat_packed must be a contiguous [{h}, w_pad] tensor, got {tuple(mat_packed.shape)}")
    if block_width <= 0 or w % block_width != 0:
        raise ValueError(f"w={w} must be divisible by N={block_width}")
    if tuple(mat_index.shape) != (w // block_width, block_width) or not mat_index.is_contiguous():
        raise ValueError(f"mat_index must be a contiguous {(w // block_width, block_width)} tensor")
    out = torch.empty((1, h), dtype=torch.float16, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(
            _lib.lib().nms_gemv_packed_f16(
                xh.data_ptr(), mat_packed.data_ptr(), mat_index.data_ptr(), out.data_ptr(),
                int(K), int(w), int(w_pad), int(h), int(block_width), int(vec_width),
                _stream_ptr(x.device),
            ),
            "nms_gemv_packed_f16",
        )
    return out.to(dtype=x.dtype).reshape(*x.shape[:-1], int(h))


@gemv_packed.register_fake
def _(x, mat_packed, mat_index, w, h, block_width, vec_width):
    return x.new_empty((*x.shape[:-1], int(h)))


_GEMM_DTYPES = {torch.float16: _lib.NMS_DTYPE_F16, torch.bfloat16: _lib.NMS_DTYPE_BF16,
                torch.float32: _lib.NMS_DTYPE_F32}


def gemm_workspace_bytes(T: int, w_pad: int, h: int) -> int:
    """Bytes of scratch nms_gemm_packed_f16 needs for T tokens (current device)."""
    n = ctypes.c_int64(0)
    _lib.check(_lib.lib().nms_gemm_workspace_bytes(int(T), int(w_pad), int(h), ctypes.byref(n)),
               "nms_gemm_workspace_bytes")
    return int(n.value)


@torch.library.custom_op("nmsparse::gemm_packed", mutates_args=())
def gemm_packed(x: torch.Tensor, mat_packed: torch.Tensor, mat_index: torch.Tensor,
                w: int, h: int, block_width: int, vec_width: int) -> torch.Tensor:
    """Shared-mask N:M product for any number of tokens (prefill / batch > 1)
    on the packed layout: every row of ``x`` [..., K] goes through the same
    sum as ``nmsparse::gemv`` (fp16 operands, fp32 accumulation, fp16
    result cast back to ``x.dtype``), on the tensor cores.  The reference
    has no multi-token sparse op; its linear falls back to a dense
    F.linear (src/spmv/nmsparse_linear.py:55-68)."""
    K = x.shape[-1]
    x2d = x.reshape(-1, K)
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    T = x2d.shape[0]
    if not x.is_cuda or not mat_packed.is_cuda or not mat_index.is_cuda:
        raise ValueError("x, mat_packed, and mat_index must be CUDA tensors")
    if x.dtype not in _GEMM_DTYPES:
        raise TypeError(f"x must be float16, bfloat16 or float32, got {x.dtype}")
    if mat_index.dtype != torch.uint8:
        raise TypeError("mat_index must be uint8")
    if mat_packed.dtype != torch.float16:
        raise TypeError("mat_packed must be float16")
    if mat_packed.ndim != 2 or mat_packed.shape[0] != h or not mat_packed.is_contiguous():
        raise ValueError(f"mat_packed must be a contiguous [{h}, w_pad] tensor, got {tuple(mat_packed.shape)}")
    if block_width <= 0 or w % block_width != 0:
        raise ValueError(f"w={w} must be divisible by N={block_width}")
    if tuple(mat_index.shape) != (w // block_width, block_width) or not mat_index.is_contiguous():
        raise ValueError(f"mat_index must be a contiguous {(w // block_width, block_width)} tensor")
    out = torch.empty((T, h), dtype=torch.float16, device=x.device)
    if T == 0:
        return out.to(dtype=x.dtype).reshape(*x.shape[:-1], int(h))
    w_pad = mat_packed.shape[-1]
    with torch.cuda.device(x.device):
        ws = torch.empty(gemm_workspace_bytes(T, w_pad, h), dtype=torch.uint8, device=x.device)
        _lib.check(
            _lib.lib().nms_gemm_packed_f16(
                x2d.data_ptr(), _GEMM_DTYPES[x.dtype], mat_packed.data_ptr(), mat_index.data_ptr(),
                out.data_ptr(), int(T), int(K), int(w), int(w_pad), int(h), int(block_width),
                int(vec_width), ws.data_ptr(), ws.numel(), _stream_ptr(x.device),
            ),
            "nms_gemm_packed_f16",
        )
    return out.to(dtype=x.dtype).reshape(*x.shape[:-1], int(h))


@gemm_packed.register_fake
def _(x, mat_packed, mat_index, w, h, block_width, vec_width):
    return x.new_empty((*x.shape[:-1], int(h)))


def pack(mat_data: torch.Tensor, w_pad: int | None = None) -> torch.Tensor:
    """Reference layout [w, h] -> packed [h, w_pad] (zero padded), bit-exact.

    CUDA tensors are converted by the library's pack kernel; CPU tensors by a
    host transpose (a one-time layout change, not the GEMV)."""
    w, h = mat_data.shape
    if w_pad is None:
        w_pad = packed_row_stride(w)
    if mat_data.dtype != torch.float16:
        raise TypeError("mat_data must be float16")
    if not mat_data.is_cuda:
        out = torch.zeros((h, w_pad), dtype=torch.float16)
        out[:, :w] = mat_data.t()
        return out
    src = mat_data.contiguous()
    out = torch.empty((h, w_pad), dtype=torch.float16, device=src.device)
    with torch.cuda.device(src.device):
        _lib.check(
            _lib.lib().nms_pack_f16(src.data_ptr(), out.data_ptr(), w, h, w_pad, _stream_ptr(src.device)),
            "nms_pack_f16",
        )
    return out


def unpack(mat_packed: torch.Tensor, w: int) -> torch.Tensor:
    """Packed [h, w_pad] -> reference layout [w, h], bit-exact."""
    h, w_pad = mat_packed.shape
    if not mat_packed.is_cuda:
        return mat_packed[:, :w].t().contiguous()
    src = mat_packed.contiguous()
    out = torch.empty((w, h), dtype=torch.float16, device=src.device)
    with torch.cuda.device(src.device):
        _lib.check(
            _lib.lib().nms_unpack_f16(src.data_ptr(), out.data_ptr(), w, h, w_pad, _stream_ptr(src.device)),
            "nms_unpack_f16",
        )
    return out


def packed_row_stride(w: int) -> int:
    """Row stride of the packed layout: w rounded up to a multiple of 64."""
    return (int(w) + 63) // 64 * 64
