"""GPU parity of the sm_100a N:M GEMV kernels against the oracle and the
reference's own outputs.

Tolerance: max-rel-error <= 1e-2 for fp16 output
against the fp32 dense product of the masked weights, where
max-rel-error = max_r |y_r - ref_r| / max_r |ref_r|.  The kernels accumulate
in fp32, so the observed error is the fp16 output rounding (~5e-4); the
tests also assert that tighter bound (2e-3) to catch real regressions.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import nm_oracle as O
from spmv_decode_b200 import _lib
from spmv_decode_b200.nmsparse_linear import NmSparseLinear, make_sparse, make_sparse_device, masked_dense
from spmv_decode_b200.nmsparse_op import pack, packed_row_stride, unpack

pytestmark = pytest.mark.gpu

TOL_MAX_REL = 1e-2
TOL_TIGHT = 2e-3
# Launches run the shared-memory ring kernel by default;
# NMS_FLAG_REGISTER_RING selects the register-ring kernel.
KERNELS = {"smem_ring": 0, "register_ring": _lib.NMS_FLAG_REGISTER_RING}

RATIOS = [(2, 4), (4, 8), (8, 16), (16, 32), (32, 64), (64, 128), (128, 256)]
SHAPES = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]  # out x in (config 2)


def _check(out: torch.Tensor, ref: np.ndarray, tol=TOL_TIGHT):
    y = out.float().reshape(-1).cpu().numpy()
    m = O.metrics(y, ref)
    assert np.isfinite(y).all()
    assert m["max_rel"] <= TOL_MAX_REL, m
    assert m["max_rel"] <= tol, m
    return m


def _oracle(x: torch.Tensor, md: torch.Tensor, mi: torch.Tensor, K: int, M: int) -> np.ndarray:
    return O.gemv_fp32(x.reshape(-1).cpu().view(torch.int16).numpy(), md.cpu().view(torch.int16).numpy(),
                       mi.cpu().numpy(), K, M)


def test_golden_reference_kernel_outputs(cuda_device):
    """Both ops reproduce the reference Triton kernel's outputs (fixtures)."""
    z = np.load(GOLDEN / "gemv.npz")
    cases = sorted({k.split("_")[0] for k in z.files if k.startswith("c")})
    for c in cases:
        K, N, M, seed, w, nnz = (int(v) for v in z[f"{c}_cfg"])
        x = torch.from_numpy(z[f"{c}_vec"]).view(torch.float16).to(cuda_device).view(1, 1, K)
        md = torch.from_numpy(z[f"{c}_mat_data"]).view(torch.float16).to(cuda_device)
        mi = torch.from_numpy(z[f"{c}_mat_index"]).to(cuda_device)
        ref = z[f"{c}_acc_generic"].reshape(-1)
        y_ref_layout = torch.ops.nmsparse.gemv(x, md, mi, w, N, nnz, M)
        assert y_ref_layout.shape == (1, 1, N) and y_ref_layout.dtype == torch.float16
        _check(y_ref_layout, ref)
        y_packed = torch.ops.nmsparse.gemv_packed(x, pack(md), mi, w, N, nnz, M)
        _check(y_packed, ref)
        # Against the reference op's own fp16 result: at most one fp16 ulp apart.
        ref16 = torch.from_numpy(z[f"{c}_op_out"]).view(torch.float16).float()
        diff = (y_ref_layout.float().cpu().reshape(-1) - ref16).abs()
        ulp = torch.clamp(ref16.abs(), min=2.0 ** -14) * 2.0 ** -10
        assert bool((diff <= ulp * 1.01).all()), c


@pytest.mark.parametrize("n,m", RATIOS)
@pytest.mark.parametrize("h,K", SHAPES)
def test_sweep_shapes_both_layouts(cuda_device, h, K, n, m):
    """Config 2 sweep: every ratio at every Llama linear shape, both layouts."""
    packed, mi, w, nnz = make_sparse_device(K, h, m, seed=h + K + m, device=cuda_device, std=0.02)
    md = unpack(packed, w)
    g = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn(1, 1, K, generator=g, device=cuda_device, dtype=torch.float32).to(torch.float16)
    ref = _oracle(x, md, mi, K, m)
    _check(torch.ops.nmsparse.gemv(x, md, mi, w, h, nnz, m), ref)
    _check(torch.ops.nmsparse.gemv_packed(x, packed, mi, w, h, nnz, m), ref)


def test_reference_packer_weights_llama_shape(cuda_device):
    """Weights from the reference-bit-exact packer at 4096x4096 32:64 (seed 0)."""
    md, mi, w, nnz = make_sparse(4096, 4096, 64, 0, "cpu")
    x = torch.randn(1, 1, 4096, generator=torch.Generator().manual_seed(0)).to(torch.float16)
    ref = _oracle(x, md, mi, 4096, 64)
    xd, mdd, mid = x.to(cuda_device), md.to(cuda_device), mi.to(cuda_device)
    _check(torch.ops.nmsparse.gemv(xd, mdd, mid, w, 4096, nnz, 64), ref)
    _check(torch.ops.nmsparse.gemv_packed(xd, pack(mdd), mid, w, 4096, nnz, 64), ref)


def test_config1_magnitude_packed_weights(cuda_device):
    """Config 1 input (W ~ N(0, 0.02) [4096, 4096], x ~ N(0, 1), 32:64) with the
    shared-mask magnitude packer; output vs fp32 masked dense product."""
    torch.manual_seed(0)
    W = (torch.randn(4096, 4096) * 0.02).to(torch.float16)
    x = torch.randn(1, 4096).to(torch.float16)
    md_np, mi_np = O.shared_mask_topk(W.view(torch.int16).numpy(), 32, 64)
    md = torch.from_numpy(md_np.view(np.int16)).view(torch.float16)
    mi = torch.from_numpy(mi_np)
    dense = O.masked_dense(md_np, mi_np, 4096, 64).astype(np.float32)
    ref = dense @ x.reshape(-1).float().numpy()
    y = torch.ops.nmsparse.gemv(x.to(cuda_device).view(1, 1, -1), md.to(cuda_device), mi.to(cuda_device),
                                2048, 4096, 32, 64)
    _check(y, ref)


@pytest.mark.parametrize("w,h", [(2, 128), (64, 100), (96, 33), (1600, 257), (896, 128), (2048, 4096), (12800, 512)])
def test_pack_unpack_roundtrip_bit_exact(cuda_device, w, h):
    md = torch.randn(w, h, device=cuda_device).to(torch.float16)
    p = pack(md)
    assert p.shape == (h, packed_row_stride(w))
    assert torch.equal(p[:, w:], torch.zeros_like(p[:, w:]))
    assert torch.equal(unpack(p, w), md)
    assert torch.equal(p.cpu(), pack(md.cpu()))


@pytest.mark.parametrize("K,h,m", [(4, 64, 4), (128, 100, 8), (192, 33, 64), (3200, 257, 32), (1792, 130, 64),
                                   (25600, 512, 32), (1024, 5, 256)])
def test_packed_edge_shapes(cuda_device, K, h, m):
    """Ragged rows, tiny widths, every lanes-per-row variant (w_pad/16 not a
    multiple of 32), and the largest K of the configs (Qwen3-32B down_proj)."""
    packed, mi, w, nnz = make_sparse_device(K, h, m, seed=K + h, device=cuda_device, std=0.05)
    x = torch.randn(1, K, device=cuda_device).to(torch.float16)
    ref = _oracle(x, unpack(packed, w), mi, K, m)
    _check(torch.ops.nmsparse.gemv_packed(x, packed, mi, w, h, nnz, m), ref)


def _fused(args, dev):
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().nms_gemv_fused_f16(ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream))


def _seg_args(segs, K, w, w_pad, n, m, x, out, epilogue=_lib.NMS_EPI_STORE):
    a = _lib.NmsGemvFusedArgs()
    for i, (p, mi) in enumerate(segs):
        a.seg[i].packed = p.data_ptr()
        a.seg[i].mat_index = None if mi is None else mi.data_ptr()
        a.seg[i].rows = p.shape[0]
    a.nseg = len(segs)
    a.epilogue = epilogue
    a.prologue = _lib.NMS_PRO_PLAIN
    a.K, a.w, a.w_pad, a.block_width, a.vec_width = K, w, w_pad, n, m
    a.x = x.data_ptr()
    a.out = out.data_ptr()
    return a


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_fused_qkv_three_masks(cuda_device, kernel):
    """q/k/v with different masks in one launch == three separate products."""
    K, m = 4096, 64
    parts = [make_sparse_device(K, r, m, seed=s, device=cuda_device, std=0.02) for r, s in
             ((4096, 1), (1024, 2), (1024, 3))]
    w, nnz = parts[0][2], parts[0][3]
    x = torch.randn(K, device=cuda_device).to(torch.float16)
    out = torch.empty(6144, device=cuda_device, dtype=torch.float16)
    a = _seg_args([(p[0], p[1]) for p in parts], K, w, parts[0][0].shape[1], nnz, m, x, out)
    a.flags = KERNELS[kernel]
    _fused(a, cuda_device)
    ref = np.concatenate([_oracle(x, unpack(p[0], w), p[1], K, m) for p in parts])
    _check(out, ref)


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_fused_swiglu_with_rmsnorm_prologue(cuda_device, kernel):
    """gate/up launch with the residual-add + RMSNorm prologue and the SwiGLU
    epilogue, against the fp16-rounding sequence of model.py:185-188, 255-270."""
    K, I, m = 4096, 14336, 64
    gate = make_sparse_device(K, I, m, seed=11, device=cuda_device, std=0.02)
    up = make_sparse_device(K, I, m, seed=12, device=cuda_device, std=0.02)
    w, nnz = gate[2], gate[3]
    xa = torch.randn(K, device=cuda_device).to(torch.float16)
    xb = torch.randn(K, device=cuda_device).to(torch.float16)
    nw = (1 + 0.1 * torch.randn(K, device=cuda_device)).to(torch.float16)
    out = torch.empty(I, device=cuda_device, dtype=torch.float16)
    resid = torch.empty(K, device=cuda_device, dtype=torch.float16)
    a = _seg_args([(gate[0], gate[1]), (up[0], up[1])], K, w, gate[0].shape[1], nnz, m, xa, out,
                  epilogue=_lib.NMS_EPI_SWIGLU)
    a.prologue = _lib.NMS_PRO_RESID_RMSNORM
    a.x2 = xb.data_ptr()
    a.norm_weight = nw.data_ptr()
    a.eps = 1e-5
    a.resid_out = resid.data_ptr()
    a.flags = KERNELS[kernel]
    _fused(a, cuda_device)
    # host restatement of the reference's roundings
    h = (xa.float() + xb.float()).to(torch.float16)
    assert torch.equal(resid, h)
    hf = h.float()
    xn = (hf * torch.rsqrt(hf.pow(2).mean() + 1e-5)).to(torch.float16)
    xn = (xn.float() * nw.float()).to(torch.float16)
    g = torch.from_numpy(_oracle(xn, unpack(gate[0], w), gate[1], K, m)).to(torch.float16)
    u = torch.from_numpy(_oracle(xn, unpack(up[0], w), up[1], K, m)).to(torch.float16)
    act = (torch.nn.functional.silu(g.float()).to(torch.float16).float() * u.float()).to(torch.float16)
    m_ = O.metrics(out.float().cpu().numpy(), act.float().numpy())
    assert m_["max_rel"] <= TOL_TIGHT, m_


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_dense_head_argmax(cuda_device, kernel):
    """Dense output head with greedy argmax epilogue, repeated launches (the
    counter resets itself), ties resolved to the lowest index."""
    V, K = 128256 // 8, 4096
    Wd = (torch.randn(V, K, device=cuda_device) * 0.02).to(torch.float16)
    x = torch.randn(K, device=cuda_device).to(torch.float16)
    logits = torch.empty(V, device=cuda_device, dtype=torch.float16)
    cap = 1024
    amax_val = torch.empty(cap, device=cuda_device, dtype=torch.float32)
    amax_idx = torch.empty(cap, device=cuda_device, dtype=torch.int32)
    counter = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    tok = torch.full((1,), -1, device=cuda_device, dtype=torch.int64)
    a = _seg_args([(Wd, None)], K, K, K, 1, 1, x, logits, epilogue=_lib.NMS_EPI_ARGMAX)
    a.flags = _lib.NMS_FLAG_DENSE | KERNELS[kernel]
    a.amax_val, a.amax_idx = amax_val.data_ptr(), amax_idx.data_ptr()
    a.amax_counter, a.token_out, a.amax_capacity = counter.data_ptr(), tok.data_ptr(), cap
    for _ in range(3):
        _fused(a, cuda_device)
    torch.cuda.synchronize()
    ref = (Wd.float() @ x.float()).cpu().numpy()
    _check(logits, ref)
    assert int(tok.item()) == int(torch.argmax(logits).item())
    assert int(counter.item()) == 0
    # force a tie: duplicate the best row further down and make it win
    best = int(tok.item())
    Wd[V - 1] = Wd[best]
    Wd[3] = Wd[best]
    _fused(a, cuda_device)
    torch.cuda.synchronize()
    assert int(tok.item()) == min(3, best)


def test_op_under_cuda_graph(cuda_device):
    md, mi, w, nnz = make_sparse(4096, 6144, 64, 3, cuda_device)
    x = torch.randn(1, 1, 4096, device=cuda_device).to(torch.float16)
    eager = torch.ops.nmsparse.gemv(x, md, mi, w, 6144, nnz, 64)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        torch.ops.nmsparse.gemv(x, md, mi, w, 6144, nnz, 64)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = torch.ops.nmsparse.gemv(x, md, mi, w, 6144, nnz, 64)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)
    assert _lib.device_error() == 0


def test_nmsparse_linear_module(cuda_device):
    """Reference constructor and attributes; packed storage holds the
    reference packer's values bit-exactly; forward == oracle; a reference
    layout state dict loads."""
    lin = NmSparseLinear(6144, 4096, 64, 5, cuda_device)
    md, mi, w, nnz = make_sparse(4096, 6144, 64, 5, "cpu")
    assert (lin.h, lin.w, lin.block_width, lin.vec_width) == (6144, w, nnz, 64)
    assert torch.equal(lin.reference_mat_data().cpu(), md)
    assert torch.equal(lin.mat_index.cpu(), mi)
    x = torch.randn(1, 1, 4096, device=cuda_device).to(torch.float16)
    _check(lin(x), _oracle(x, md, mi, 4096, 64))
    lin2 = NmSparseLinear(6144, 4096, 64, 99, cuda_device)
    lin2.load_state_dict({"mat_data": md.to(cuda_device), "mat_index": mi.to(cuda_device)}, strict=False)
    assert torch.equal(lin2.mat_data, lin.mat_data)
    assert torch.equal(lin2(x), lin(x))



@pytest.mark.parametrize("kernel", sorted(KERNELS))
@pytest.mark.parametrize("grid", [0, 1, 37, 148, 296])
@pytest.mark.parametrize("K,h,m", [(4096, 6144, 64), (14336, 4096, 16), (3200, 257, 32), (896, 130, 64)])
def test_grid_sizes_and_pdl(cuda_device, grid, K, h, m, kernel):
    """Any CTA count (row ranges split unevenly, one CTA doing everything)
    matches the oracle, with and without programmatic dependent launch."""
    packed, mi, w, nnz = make_sparse_device(K, h, m, seed=K * 3 + h, device=cuda_device, std=0.03)
    x = torch.randn(K, device=cuda_device).to(torch.float16)
    ref = _oracle(x, unpack(packed, w), mi, K, m)
    for pdl in (0, _lib.NMS_FLAG_PDL):
        out = torch.full((h,), float("nan"), device=cuda_device, dtype=torch.float16)
        a = _seg_args([(packed, mi)], K, w, packed.shape[1], nnz, m, x, out)
        a.flags = pdl | KERNELS[kernel]
        a.grid = grid
        _fused(a, cuda_device)
        _check(out, ref)


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_fused_swiglu_plain_prologue(cuda_device, kernel):
    """gate/up with the SwiGLU epilogue on an already-normalised input (plain
    prologue: the shared-memory ring kernel by default)."""
    K, I, m = 4096, 14336, 64
    gate = make_sparse_device(K, I, m, seed=21, device=cuda_device, std=0.02)
    up = make_sparse_device(K, I, m, seed=22, device=cuda_device, std=0.02)
    w, nnz = gate[2], gate[3]
    x = torch.randn(K, device=cuda_device).to(torch.float16)
    out = torch.empty(I, device=cuda_device, dtype=torch.float16)
    a = _seg_args([(gate[0], gate[1]), (up[0], up[1])], K, w, gate[0].shape[1], nnz, m, x, out,
                  epilogue=_lib.NMS_EPI_SWIGLU)
    a.flags = KERNELS[kernel]
    _fused(a, cuda_device)
    g = torch.from_numpy(_oracle(x, unpack(gate[0], w), gate[1], K, m)).to(torch.float16)
    u = torch.from_numpy(_oracle(x, unpack(up[0], w), up[1], K, m)).to(torch.float16)
    act = (torch.nn.functional.silu(g.float()).to(torch.float16).float() * u.float()).to(torch.float16)
    m_ = O.metrics(out.float().cpu().numpy(), act.float().numpy())
    assert m_["max_rel"] <= TOL_TIGHT, m_


@pytest.mark.parametrize("n,m", [(2, 4), (16, 32), (32, 64), (128, 256)])
def test_ring_kernel_pdl_chain_in_graph(cuda_device, n, m):
    """Back-to-back dependent launches (each GEMV reads the previous one's
    output) with programmatic dependent launch in a CUDA graph: the shared-
    memory ring kernel lets its dependents start at once and fills their
    rings early, so this checks that every launch still reads its input only
    after its producer finished.  Each stage against the oracle on the
    previous stage's fp16 output; replays bit-identical."""
    K = 4096
    stages = [make_sparse_device(K, K, m, seed=40 + i, device=cuda_device, std=1.0 / 64) for i in range(6)]
    w, nnz = stages[0][2], stages[0][3]
    x0 = torch.randn(K, device=cuda_device).to(torch.float16)
    bufs = [x0] + [torch.empty(K, device=cuda_device, dtype=torch.float16) for _ in stages]
    args = []
    for i, (p, mi, _, _) in enumerate(stages):
        a = _seg_args([(p, mi)], K, w, p.shape[1], nnz, m, bufs[i], bufs[i + 1])
        a.flags = _lib.NMS_FLAG_PDL
        args.append(a)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        for a in args:
            _lib.check(_lib.lib().nms_gemv_fused_f16(ctypes.byref(a), s.cuda_stream))
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    torch.cuda.synchronize(cuda_device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for a in args:
            _lib.check(_lib.lib().nms_gemv_fused_f16(ctypes.byref(a), s.cuda_stream))
    for b in bufs[1:]:
        b.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize(cuda_device)
    first = [b.clone() for b in bufs[1:]]
    for i, (p, mi, _, _) in enumerate(stages):
        _check(bufs[i + 1], _oracle(bufs[i], unpack(p, w), mi, K, m))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(cuda_device)
    for b, f in zip(bufs[1:], first):
        assert torch.equal(b, f)
    assert _lib.device_error() == 0
