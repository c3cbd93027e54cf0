"""ctypes binding of libnmsparse_b200.so (the C ABI declared in
include/nmsparse_b200.h).

The library is built in-tree by ``spmv_decode_b200.build`` into
``spmv_decode_b200/lib/libnmsparse_b200.so``.  There is no fallback: if the
library is missing, every entry point raises ``RuntimeError`` naming the
build command.  Status codes map to the exception types the reference raises
for the same conditions (triton_spmv.py:245-283; src/spmv/nmsparse_op.py:84-87).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libnmsparse_b200.so"

NMS_OK = 0
NMS_ERR_VALUE = -1
NMS_ERR_TYPE = -2
NMS_ERR_NOT_IMPLEMENTED = -3
NMS_ERR_CUDA = -4
NMS_ERR_DEVICE = -5

ABI_VERSION = 2  # NMS_ABI_VERSION of include/nmsparse_b200.h these declarations match
NMS_MAX_SEGMENTS = 4
NMS_EPI_STORE = 0
NMS_EPI_SWIGLU = 1
NMS_EPI_ARGMAX = 2
NMS_PRO_PLAIN = 0
NMS_PRO_RESID_RMSNORM = 1
NMS_FLAG_PDL = 1
NMS_FLAG_DENSE = 2
NMS_FLAG_REGISTER_RING = 4
NMS_ROPE_INTERLEAVED = 0
NMS_ROPE_HALF = 1
NMS_DTYPE_F16 = 0
NMS_DTYPE_BF16 = 1
NMS_DTYPE_F32 = 2

# Every exported symbol of include/nmsparse_b200.h (checked by the CPU tests).
EXPORTED_SYMBOLS = (
    "nms_abi_version",
    "nms_source_hash",
    "nms_device_error_set",
    "nms_step_reset",
    "nms_last_error",
    "nms_status_name",
    "nms_num_sms",
    "nms_device_error",
    "nms_gemv_f16",
    "nms_gemv_rowwise_f16",
    "nms_gemm_workspace_bytes",
    "nms_gemm_packed_f16",
    "nms_packed_row_stride",
    "nms_pack_f16",
    "nms_unpack_f16",
    "nms_gemv_packed_f16",
    "nms_gemv_fused_f16",
    "nms_attention_decode_f16",
    "nms_embedding_f16",
    "nms_gemv_argmax_noalloc_f16",
    "nms_plan_create",
    "nms_plan_destroy",
    "nms_plan_add_gemv",
    "nms_plan_add_attention",
    "nms_plan_add_embedding",
    "nms_plan_size",
    "nms_plan_launch",
    "nms_step_create",
    "nms_step_create_flow",
    "nms_step_launch",
    "nms_step_destroy",
    "nms_step_info",
    "nms_step_set_trace",
    "nms_tp_area_bytes",
    "nms_ipc_alloc",
    "nms_ipc_free",
    "nms_ipc_open",
    "nms_ipc_close",
    "nms_step_set_tp",
)

NMS_MAX_TP = 8


class NmsTpConfig(ctypes.Structure):
    """nms_tp_config (include/nmsparse_b200.h)."""

    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("vocab_offset", ctypes.c_int32), ("area", ctypes.c_void_p * NMS_MAX_TP)]


c_void_p = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64


class NmsSegment(ctypes.Structure):
    _fields_ = [("packed", c_void_p), ("mat_index", c_void_p), ("rows", c_i64)]


class NmsGemvFusedArgs(ctypes.Structure):
    _fields_ = [
        ("seg", NmsSegment * NMS_MAX_SEGMENTS),
        ("nseg", c_i32),
        ("epilogue", c_i32),
        ("prologue", c_i32),
        ("flags", c_i32),
        ("K", c_i64),
        ("w", c_i64),
        ("w_pad", c_i64),
        ("block_width", c_i32),
        ("vec_width", c_i32),
        ("x", c_void_p),
        ("x2", c_void_p),
        ("norm_weight", c_void_p),
        ("eps", ctypes.c_float),
        ("resid_out", c_void_p),
        ("out", c_void_p),
        ("amax_val", c_void_p),
        ("amax_idx", c_void_p),
        ("amax_counter", c_void_p),
        ("token_out", c_void_p),
        ("amax_capacity", c_i32),
        ("grid", c_i32),
        ("prefetch_bytes", c_i32),
        ("next_token", c_void_p),
        ("token_history", c_void_p),
        ("pos", c_void_p),
        ("history_len", c_i64),
        ("next_prefetch", c_void_p * 2),
        ("next_prefetch_bytes", c_i64 * 2),
        ("next_prefetch_head", c_i64),
        ("x_token", c_void_p),
        ("x_rows", c_i64),
        ("temperature", ctypes.c_float),
        ("sample_seed", ctypes.c_uint64),
        ("sample_pos", c_void_p),
        ("sample_row_offset", c_i64),
    ]


class NmsAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", c_void_p),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
        ("rope", c_void_p),
        ("q_norm", c_void_p),
        ("k_norm", c_void_p),
        ("pos", c_void_p),
        ("y", c_void_p),
        ("Hq", c_i32),
        ("Hkv", c_i32),
        ("D", c_i32),
        ("S_max", c_i32),
        ("rope_style", c_i32),
        ("splits", c_i32),
        ("norm_eps", ctypes.c_float),
        ("scale", ctypes.c_float),
        ("flags", c_i32),
        ("next_prefetch", c_void_p * 2),
        ("next_prefetch_bytes", c_i64 * 2),
        ("next_prefetch_head", c_i64),
    ]


_LIB = None


def _declare(lib: ctypes.CDLL) -> None:
    P, I32, I64 = c_void_p, c_i32, c_i64
    sig = {
        "nms_abi_version": (I32, []),
        "nms_source_hash": (ctypes.c_char_p, []),
        "nms_device_error_set": (I32, [I32]),
        "nms_step_reset": (I32, [P, P]),
        "nms_last_error": (ctypes.c_char_p, []),
        "nms_status_name": (ctypes.c_char_p, [I32]),
        "nms_num_sms": (I32, [ctypes.POINTER(I32)]),
        "nms_device_error": (I32, [ctypes.POINTER(I32), I32]),
        "nms_gemv_f16": (I32, [P, P, P, P, I64, I64, I64, I32, I32, P]),
        "nms_gemv_rowwise_f16": (I32, [P, P, P, P, I64, I64, I64, I32, I32, P]),
        "nms_gemm_workspace_bytes": (I32, [I64, I64, I64, ctypes.POINTER(c_i64)]),
        "nms_gemm_packed_f16": (I32, [P, I32, P, P, P, I64, I64, I64, I64, I64, I32, I32, P, I64, P]),
        "nms_packed_row_stride": (I64, [I64]),
        "nms_pack_f16": (I32, [P, P, I64, I64, I64, P]),
        "nms_unpack_f16": (I32, [P, P, I64, I64, I64, P]),
        "nms_gemv_packed_f16": (I32, [P, P, P, P, I64, I64, I64, I64, I32, I32, P]),
        "nms_gemv_fused_f16": (I32, [ctypes.POINTER(NmsGemvFusedArgs), P]),
        "nms_attention_decode_f16": (I32, [ctypes.POINTER(NmsAttentionArgs), P]),
        "nms_embedding_f16": (I32, [P, P, P, I64, I64, I32, P]),
        "nms_gemv_argmax_noalloc_f16": (I32, [P, P, P, ctypes.c_float, P, I64, I64, P, P, P]),
        "nms_plan_create": (I32, [ctypes.POINTER(P)]),
        "nms_plan_destroy": (I32, [P]),
        "nms_plan_add_gemv": (I32, [P, ctypes.POINTER(NmsGemvFusedArgs)]),
        "nms_plan_add_attention": (I32, [P, ctypes.POINTER(NmsAttentionArgs)]),
        "nms_plan_add_embedding": (I32, [P, P, P, P, I64, I64, I32]),
        "nms_plan_size": (I32, [P, ctypes.POINTER(I32)]),
        "nms_plan_launch": (I32, [P, I32, I32, P]),
        "nms_step_create": (I32, [P, ctypes.POINTER(I32), I32, ctypes.POINTER(P)]),
        "nms_step_create_flow": (I32, [P, ctypes.POINTER(I32), I32, ctypes.POINTER(P)]),
        "nms_step_launch": (I32, [P, P]),
        "nms_step_destroy": (I32, [P]),
        "nms_step_info": (I32, [P, ctypes.POINTER(I32), ctypes.POINTER(I32)]),
        "nms_step_set_trace": (I32, [P, P, I64]),
        "nms_tp_area_bytes": (I64, [I32, I32, I32]),
        "nms_ipc_alloc": (I32, [I64, ctypes.POINTER(P), P]),
        "nms_ipc_free": (I32, [P]),
        "nms_ipc_open": (I32, [P, ctypes.POINTER(P)]),
        "nms_ipc_close": (I32, [P]),
        "nms_step_set_tp": (I32, [P, ctypes.POINTER(I32), I32, ctypes.POINTER(NmsTpConfig)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """Load (once) and return the C library; raise if it was not built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"libnmsparse_b200.so not found at {LIB_PATH}; build it with "
                "`python -c 'import spmv_decode_b200.build as b; b.build()'` "
                "(there is no CPU or Triton fallback)"
            )
        mode = os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0)
        handle = ctypes.CDLL(str(LIB_PATH), mode=mode)
        _declare(handle)
        if handle.nms_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH} has ABI {handle.nms_abi_version()}, these bindings expect {ABI_VERSION}; "
                               "rebuild it with `python -m spmv_decode_b200.build`")
        _LIB = handle
    return _LIB


_EXC = {
    NMS_ERR_VALUE: ValueError,
    NMS_ERR_TYPE: TypeError,
    NMS_ERR_NOT_IMPLEMENTED: NotImplementedError,
}


def check(rc: int, what: str = "") -> None:
    """Raise the exception mapped from a nonzero nms_status."""
    if rc == NMS_OK:
        return
    L = lib()
    msg = L.nms_last_error().decode(errors="replace")
    name = L.nms_status_name(rc).decode()
    exc = _EXC.get(rc, RuntimeError)
    prefix = f"{what}: " if what else ""
    raise exc(f"{prefix}{msg} [{name}]")


def num_sms() -> int:
    v = c_i32(0)
    check(lib().nms_num_sms(ctypes.byref(v)), "nms_num_sms")
    return int(v.value)


def device_error(clear: bool = True) -> int:
    v = c_i32(0)
    check(lib().nms_device_error(ctypes.byref(v), 1 if clear else 0), "nms_device_error")
    return int(v.value)


def source_hash() -> str:
    """SHA-256 of the sources the loaded library was built from."""
    return lib().nms_source_hash().decode()


def packed_row_stride(w: int) -> int:
    return int(lib().nms_packed_row_stride(int(w)))


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
