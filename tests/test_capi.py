"""The C-ABI library loads, exports every declared symbol, and rejects bad
arguments with the mapped exception types -- all without a GPU (argument
validation runs before any CUDA call)."""
import ctypes
import re

import pytest
import torch

from conftest import ROOT
from spmv_decode_b200 import _lib
from spmv_decode_b200.nmsparse_op import packed_row_stride

HEADER = ROOT / "include" / "nmsparse_b200.h"


def _declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nms_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    assert sorted(_lib.EXPORTED_SYMBOLS) == declared
    for name in declared:
        assert hasattr(L, name), name
    assert L.nms_abi_version() == _lib.ABI_VERSION == 2


def test_status_names():
    L = _lib.lib()
    assert L.nms_status_name(0) == b"NMS_OK"
    assert L.nms_status_name(-1) == b"NMS_ERR_VALUE"
    assert L.nms_status_name(-3) == b"NMS_ERR_NOT_IMPLEMENTED"


def test_packed_row_stride_matches_python():
    for w in (1, 2, 63, 64, 65, 896, 1600, 2048, 7168, 12800):
        assert _lib.packed_row_stride(w) == packed_row_stride(w)
        assert packed_row_stride(w) % 64 == 0 and packed_row_stride(w) >= w


def _call_gemv(**kw):
    a = dict(vec=1, mat_data=32, mat_index=1, out=1, K=4096, w=2048, h=4096, bw=32, vw=64)
    a.update(kw)
    return _lib.lib().nms_gemv_f16(a["vec"], a["mat_data"], a["mat_index"], a["out"], a["K"], a["w"], a["h"],
                                   a["bw"], a["vw"], None)


@pytest.mark.parametrize(
    "kw,msg",
    [
        (dict(vec=None), "null pointer"),
        (dict(h=4000), "divisible by 128"),
        (dict(w=2047), "divisible by N"),
        (dict(K=4000), "K=4000"),
        (dict(bw=0), "positive"),
        (dict(bw=64, vw=32), "must not exceed"),
        (dict(vw=512, bw=256, w=2048, K=4096), "uint8"),
        (dict(mat_data=34), "32-byte aligned"),
    ],
)
def test_gemv_argument_validation(kw, msg):
    rc = _call_gemv(**kw)
    assert rc == _lib.NMS_ERR_VALUE
    assert msg in _lib.lib().nms_last_error().decode()
    with pytest.raises(ValueError, match=re.escape(msg)):
        _lib.check(rc)


def test_fused_argument_validation():
    a = _lib.NmsGemvFusedArgs()
    a.nseg = 0
    rc = _lib.lib().nms_gemv_fused_f16(ctypes.byref(a), None)
    assert rc == _lib.NMS_ERR_VALUE
    a.nseg = 2
    a.x = 16
    a.out = 16
    a.epilogue = _lib.NMS_EPI_SWIGLU
    a.K, a.w, a.w_pad, a.block_width, a.vec_width = 4096, 2048, 2048, 32, 64
    a.seg[0].packed, a.seg[0].mat_index, a.seg[0].rows = 32, 16, 128
    a.seg[1].packed, a.seg[1].mat_index, a.seg[1].rows = None, 16, 128
    rc = _lib.lib().nms_gemv_fused_f16(ctypes.byref(a), None)
    assert rc == _lib.NMS_ERR_VALUE  # null segment pointer is rejected before any CUDA call
    a.seg[1].packed = 64
    a.epilogue = 7
    assert _lib.lib().nms_gemv_fused_f16(ctypes.byref(a), None) == _lib.NMS_ERR_VALUE
    assert "unknown epilogue" in _lib.lib().nms_last_error().decode()


def test_attention_argument_validation():
    a = _lib.NmsAttentionArgs()
    rc = _lib.lib().nms_attention_decode_f16(ctypes.byref(a), None)
    assert rc == _lib.NMS_ERR_VALUE
    a.qkv = a.k_cache = a.v_cache = a.rope = a.pos = a.y = 256
    a.D = 64
    rc = _lib.lib().nms_attention_decode_f16(ctypes.byref(a), None)
    assert rc == _lib.NMS_ERR_NOT_IMPLEMENTED
    with pytest.raises(NotImplementedError):
        _lib.check(rc)


def test_plan_lifecycle_without_gpu():
    L = _lib.lib()
    h = ctypes.c_void_p()
    assert L.nms_plan_create(ctypes.byref(h)) == 0
    n = ctypes.c_int32(-1)
    assert L.nms_plan_size(h, ctypes.byref(n)) == 0 and n.value == 0
    assert L.nms_plan_launch(h, 0, 1, None) == _lib.NMS_ERR_VALUE  # range outside an empty plan
    assert L.nms_plan_add_embedding(h, None, None, None, 16, 16, 0) == _lib.NMS_ERR_VALUE
    assert L.nms_plan_destroy(h) == 0


def test_op_rejects_cpu_tensors_like_the_reference():
    """Reference wrapper: ValueError for non-CUDA tensors (triton_spmv.py:245-246)."""
    from spmv_decode_b200 import nmsparse_op  # noqa: F401

    x = torch.randn(1, 1, 256, dtype=torch.float16)
    md = torch.zeros(128, 128, dtype=torch.float16)
    mi = torch.zeros(8, 16, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA tensors"):
        torch.ops.nmsparse.gemv(x, md, mi, 128, 128, 16, 32)
    with pytest.raises(RuntimeError, match="rows==1"):
        torch.ops.nmsparse.gemv(torch.randn(1, 2, 256, dtype=torch.float16), md, mi, 128, 128, 16, 32)


def test_fake_kernel_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(1, 1, 512, dtype=torch.float16)
        md = torch.empty(256, 384, dtype=torch.float16)
        mi = torch.empty(16, 16, dtype=torch.uint8)
        y = torch.ops.nmsparse.gemv(x, md, mi, 256, 384, 16, 32)
        assert tuple(y.shape) == (1, 1, 384)


def _call_gemm(**kw):
    a = dict(x=256, dt=_lib.NMS_DTYPE_F16, packed=256, mi=256, out=256, T=128, K=4096, w=2048, w_pad=2048, h=4096,
             bw=32, vw=64, ws=256, wsb=1 << 30)
    a.update(kw)
    return _lib.lib().nms_gemm_packed_f16(a["x"], a["dt"], a["packed"], a["mi"], a["out"], a["T"], a["K"], a["w"],
                                          a["w_pad"], a["h"], a["bw"], a["vw"], a["ws"], a["wsb"], None)


@pytest.mark.parametrize(
    "kw,status,msg",
    [
        (dict(x=None), _lib.NMS_ERR_VALUE, "null pointer"),
        (dict(ws=None), _lib.NMS_ERR_VALUE, "null pointer"),
        (dict(dt=7), _lib.NMS_ERR_TYPE, "x_dtype=7"),
        (dict(T=0), _lib.NMS_ERR_VALUE, "T=0"),
        (dict(K=4000), _lib.NMS_ERR_VALUE, "K=4000"),
        (dict(w=2047), _lib.NMS_ERR_VALUE, "divisible by N"),
        (dict(w_pad=2050), _lib.NMS_ERR_VALUE, "w_pad=2050"),
        (dict(bw=64, vw=32), _lib.NMS_ERR_VALUE, "N <= M"),
        (dict(packed=264), _lib.NMS_ERR_VALUE, "16-byte aligned"),
        (dict(ws=272), _lib.NMS_ERR_VALUE, "256-byte aligned"),
        (dict(x=257), _lib.NMS_ERR_VALUE, "element size"),
    ],
)
def test_gemm_argument_validation(kw, status, msg):
    """The prefill GEMM validates every argument before touching the device."""
    rc = _call_gemm(**kw)
    assert rc == status
    assert msg in _lib.lib().nms_last_error().decode()


def test_gemm_op_rejects_cpu_tensors():
    from spmv_decode_b200 import nmsparse_op  # noqa: F401

    x = torch.randn(4, 256, dtype=torch.float16)
    packed = torch.zeros(128, 128, dtype=torch.float16)
    mi = torch.zeros(8, 16, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA tensors"):
        torch.ops.nmsparse.gemm_packed(x, packed, mi, 128, 128, 16, 32)
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        y = torch.ops.nmsparse.gemm_packed(torch.empty(3, 5, 256, dtype=torch.bfloat16),
                                           torch.empty(384, 128, dtype=torch.float16),
                                           torch.empty(8, 16, dtype=torch.uint8), 128, 384, 16, 32)
        assert tuple(y.shape) == (3, 5, 384) and y.dtype == torch.bfloat16


@pytest.mark.parametrize("T,w_pad,h,msg", [(0, 2048, 4096, "positive"), (16, 2000, 4096, "multiple of 64"),
                                           (16, 2048, 0, "positive")])
def test_gemm_workspace_argument_validation(T, w_pad, h, msg):
    n = ctypes.c_int64(-1)
    rc = _lib.lib().nms_gemm_workspace_bytes(T, w_pad, h, ctypes.byref(n))
    assert rc == _lib.NMS_ERR_VALUE and n.value == -1
    assert msg in _lib.lib().nms_last_error().decode()
    assert _lib.lib().nms_gemm_workspace_bytes(16, 2048, 4096, None) == _lib.NMS_ERR_VALUE


def _call_noalloc(x=1, x2=None, norm=None, head=1, vocab=128, K=64, logits=1, token=1):
    L = _lib.lib()
    tok = ctypes.c_int64(0) if token else None
    return L.nms_gemv_argmax_noalloc_f16(x, x2, norm, ctypes.c_float(1e-5), head, vocab, K, logits,
                                         ctypes.byref(tok) if tok is not None else None, None)


@pytest.mark.parametrize("kw, msg", [
    (dict(x=None), "null pointer"),
    (dict(head=None), "null pointer"),
    (dict(logits=None), "null pointer"),
    (dict(token=None), "null pointer"),
    (dict(K=96), "multiple of 64"),
    (dict(K=0), "multiple of 64"),
    (dict(vocab=0), "out of range"),
    (dict(vocab=(1 << 30) + 1), "out of range"),
])
def test_noalloc_head_argument_validation(kw, msg):
    """nms_gemv_argmax_noalloc_f16 rejects bad arguments before any CUDA call."""
    rc = _call_noalloc(**kw)
    assert rc == _lib.NMS_ERR_VALUE
    assert msg in _lib.lib().nms_last_error().decode()


def test_device_error_set_rejects_non_positive_codes():
    L = _lib.lib()
    for code in (0, -3):
        assert L.nms_device_error_set(code) == _lib.NMS_ERR_VALUE
        assert "positive" in L.nms_last_error().decode()


def test_step_reset_rejects_null():
    assert _lib.lib().nms_step_reset(None, None) == _lib.NMS_ERR_VALUE


def test_library_source_hash_matches_tree():
    """The loaded library was built from the sources in this tree."""
    from spmv_decode_b200 import build

    assert _lib.source_hash() == build.source_hash()
