"""N:M sparse GEMV microbenchmark (the reference's
``microbench_triton_torchmv.py`` measures the same shapes and ratios).

    python -m spmv_decode_b200.microbench [--ratios 2:4,...] [--shapes 6144x4096,...] [--reps 20]

For every shape (out x in) and N:M ratio: seeded synthetic shared-mask weights
(N(0, 0.02) values, uniform random in-group masks, drawn on the GPU), a vector
~N(0, 1); the time of one launch of

* ``packed``   -- ``nms_gemv_packed_f16`` on the re-laid-out packed weights
                  (the kernel behind ``nmsparse::gemv_packed`` / NmSparseLinear:
                  ``gemv_ring_kernel``, per-warp shared-memory weight rings);
                  ``packed_pdl``: the same launches with programmatic
                  dependent launch, as the decode plan issues them;
                  ``regring_pdl``: ``gemv_packed_kernel`` (register-ring
                  streaming, ``NMS_FLAG_REGISTER_RING``) with PDL;
* ``step``     -- the same GEMV as a one-stage launch of the persistent
                  decode-step kernel (per-warp shared-memory weight rings);
* ``ref``      -- ``gemv_ref_kernel`` on the reference ``[w, h]`` layout
                  (the kernel behind ``nmsparse::gemv``);
* ``cublas``   -- dense fp16 ``torch.mv`` (cuBLAS) on a dense matrix of the
                  same shape (the control);
* ``rowwise``  -- the per-row layout (top-|w| per row and
                  group, one uint8 offset per kept value) at 32:64;
* ``triton_ref`` (``--triton-ref``) -- the reference's own Triton kernel,
                  ``nmsparse_spmv_forward_triton_ptx`` (triton_spmv.py:229-318:
                  fp32 zero-fill, ``nmsparse_generic_kernel`` on this GPU --
                  the A100 variant is gated to sm80/sm86, :222-226 -- and the
                  fp16 cast), unmodified, imported from the reference install
                  in ``baseline/_ref``; a comparison arm only, nothing in the
                  library imports it;

``--gemm 16,128,...`` instead times the prefill / batch > 1 GEMM
(``nmsparse::gemm_packed``: gather + tcgen05 GEMM) against cuBLAS dense
``F.linear`` for each token count and shape, with its roofline fraction
(max of the HBM time and the tensor time of the sparse FLOPs).

Each of the above runs as a CUDA graph of back-to-back launches over enough weight copies to
span more than 3x the 126 MB L2 (so every launch streams from HBM), timed with
CUDA events.  Achieved bandwidth = algorithmic bytes (kept values + mask
offsets + vector + output; dense: the full matrix) / time, also as a fraction
of the measured HBM copy bandwidth (MEASURED_PEAKS.json when present).  Each
kernel's output is checked against the fp32 product of the masked dense matrix
(max-rel-error, the reference microbench's metric).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
from pathlib import Path

import torch

from . import _lib
from .nmsparse_linear import make_sparse_device, masked_dense
from .nmsparse_op import unpack

L2_BYTES = 126 * 2 ** 20
SHAPES = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]
RATIOS = [(2, 4), (4, 8), (8, 16), (16, 32), (32, 64), (64, 128), (128, 256)]


def _peak_tflops() -> tuple:
    """Dense fp16/bf16 tensor peak (the burst cuBLAS figure), TFLOP/s."""
    f = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def _peak_gbs() -> tuple:
    f = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        for k in ("hbm_gbs", "hbm_copy_gbs"):
            if k in d:
                return float(d[k]), "measured"
    return 6650.0, "fallback"


def _graph_time_us(fns, dev, reps: int) -> float:
    """Mean time of one call of ``fns`` (captured back-to-back in a graph)."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for f in fns:
            f(s)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f(s)
    cur = torch.cuda.current_stream(dev)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    del g
    return e0.elapsed_time(e1) * 1e3 / reps / len(fns)


def _max_rel(y: torch.Tensor, ref: torch.Tensor) -> float:
    return float((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def _triton_reference():
    """The reference's Triton GEMV module from ``baseline/_ref`` (None, reason)
    when it is not installed or does not import."""
    import sys

    ref_dir = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (ref_dir / "triton_spmv.py").exists():
        return None, f"reference not installed in {ref_dir}"
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    try:
        import triton_spmv  # noqa: the reference's module, unmodified
    except Exception as exc:  # reported, not required
        return None, f"{type(exc).__name__}: {exc}"[:300]
    return triton_spmv, None


def bench_shape(h: int, K: int, ratios, dev, reps: int, peak: float, triton_ref: bool = False) -> list:
    lib = _lib.lib()
    rows = []
    x = torch.randn(K, device=dev, generator=torch.Generator(device=dev).manual_seed(1)).to(torch.float16)
    # Dense cuBLAS control.
    dense_bytes = h * K * 2 + K * 2 + h * 2
    nb = max(2, math.ceil(3 * L2_BYTES / dense_bytes) + 1)
    Ws = [(torch.randn(h, K, device=dev) * 0.02).to(torch.float16) for _ in range(nb)]
    outs = [torch.empty(h, device=dev, dtype=torch.float16) for _ in range(nb)]
    t_dense = _graph_time_us([(lambda i: lambda s: torch.mv(Ws[i], x, out=outs[i]))(i) for i in range(nb)], dev,
                             reps)
    del Ws, outs
    torch.cuda.empty_cache()
    for (n, m) in ratios:
        if K % m:
            continue
        w = K // m * n
        alg = h * w * 2 + w + K * 2 + h * 2
        nb = max(2, math.ceil(3 * L2_BYTES / alg) + 1)
        mats = [make_sparse_device(K, h, m, seed=i, device=dev, std=0.02) for i in range(nb)]
        outs = [torch.empty(h, device=dev, dtype=torch.float16) for _ in range(nb)]

        def packed_fn(i):
            p, mi, w_, nnz = mats[i]
            return lambda s: _lib.check(lib.nms_gemv_packed_f16(x.data_ptr(), p.data_ptr(), mi.data_ptr(),
                                                                outs[i].data_ptr(), K, w_, p.shape[1], h, nnz, m,
                                                                s.cuda_stream), "nms_gemv_packed_f16")

        t_packed = _graph_time_us([packed_fn(i) for i in range(nb)], dev, reps)
        # Back-to-back launches with programmatic dependent launch (as in the
        # decode step's plan): a launch's first weight loads overlap the
        # previous launch's tail.
        fargs = []
        for i in range(nb):
            p_, mi_, w_, nnz_ = mats[i]
            a = _lib.NmsGemvFusedArgs()
            a.seg[0].packed, a.seg[0].mat_index, a.seg[0].rows = p_.data_ptr(), mi_.data_ptr(), h
            a.nseg, a.flags = 1, _lib.NMS_FLAG_PDL
            a.K, a.w, a.w_pad, a.block_width, a.vec_width = K, w_, p_.shape[1], nnz_, m
            a.x, a.out = x.data_ptr(), outs[i].data_ptr()
            fargs.append(a)
        t_pdl = _graph_time_us([(lambda a: lambda s: _lib.check(lib.nms_gemv_fused_f16(ctypes.byref(a), s.cuda_stream)))(a)
                                for a in fargs], dev, reps)
        for a in fargs:
            a.flags = _lib.NMS_FLAG_PDL | _lib.NMS_FLAG_REGISTER_RING
        outs[0].zero_()
        t_reg = _graph_time_us([(lambda a: lambda s: _lib.check(lib.nms_gemv_fused_f16(ctypes.byref(a), s.cuda_stream)))(a)
                                for a in fargs], dev, reps)
        p0_, mi0_, _, _ = mats[0]
        reg_err = _max_rel(outs[0], masked_dense(unpack(p0_, w), mi0_, K, m).float() @ x.float())
        for a in fargs:
            a.flags = _lib.NMS_FLAG_PDL
        p0, mi0, _, _ = mats[0]
        ref = masked_dense(unpack(p0, w), mi0, K, m).float() @ x.float()
        packed_err = _max_rel(outs[0], ref)
        # The GEMV as one stage of the persistent decode-step kernel (per-warp
        # shared-memory weight rings filled before the predecessor is waited
        # for), one cooperative launch per GEMV.
        steps = []
        plan = ctypes.c_void_p()
        _lib.check(lib.nms_plan_create(ctypes.byref(plan)))
        for a in fargs:
            _lib.check(lib.nms_plan_add_gemv(plan, ctypes.byref(a)))
        for i in range(nb):
            st = ctypes.c_void_p()
            rec = (ctypes.c_int32 * 1)(i)
            _lib.check(lib.nms_step_create(plan, rec, 1, ctypes.byref(st)), "nms_step_create")
            steps.append(st)
        outs[0].zero_()
        t_step = _graph_time_us([(lambda st: lambda s: _lib.check(lib.nms_step_launch(st, s.cuda_stream)))(st)
                                 for st in steps], dev, reps)
        step_err = _max_rel(outs[0], ref)
        for st in steps:
            lib.nms_step_destroy(st)
        lib.nms_plan_destroy(plan)
        # Reference [w, h] layout (h % 128 == 0, as the reference requires).
        refm = [unpack(mats[i][0], w) for i in range(nb)]
        del mats
        torch.cuda.empty_cache()

        def ref_fn(i):
            return lambda s: _lib.check(lib.nms_gemv_f16(x.data_ptr(), refm[i].data_ptr(), mi0.data_ptr(),
                                                         outs[i].data_ptr(), K, w, h, n, m, s.cuda_stream),
                                        "nms_gemv_f16")

        # every copy shares mask 0 here: the kernel's bytes and access pattern do not depend on the mask
        t_ref = _graph_time_us([ref_fn(i) for i in range(nb)], dev, reps)
        ref_err = _max_rel(outs[0], masked_dense(refm[0], mi0, K, m).float() @ x.float())
        tri = {}
        if triton_ref:
            mod, why = _triton_reference()
            if mod is None:
                tri = {"triton_ref_error": why}
            else:
                vec = x.view(1, K)
                ys = [None] * nb

                def tri_fn(i):
                    def f(s):
                        ys[i] = mod.nmsparse_spmv_forward_triton_ptx(vec, refm[i], mi0, w, h, n, 128, m, 1, K)
                    return f

                try:
                    t_tri = _graph_time_us([tri_fn(i) for i in range(nb)], dev, reps)
                    tri_fn(0)(None)
                    torch.cuda.synchronize(dev)
                    tri = {"triton_ref_us": round(t_tri, 3), "triton_ref_GBs": round(alg / t_tri / 1e3, 1),
                           "triton_ref_frac": round(alg / t_tri / 1e3 / peak, 3),
                           "triton_ref_max_rel": _max_rel(ys[0].view(-1), masked_dense(refm[0], mi0, K, m).float()
                                                          @ x.float()),
                           "speedup_vs_triton_ref": round(t_tri / t_packed, 3)}
                except Exception as exc:
                    tri = {"triton_ref_error": f"{type(exc).__name__}: {exc}"[:300]}
                del ys
        del refm, outs
        torch.cuda.empty_cache()
        rows.append({
            "shape": f"{h}x{K}", "nm": f"{n}:{m}", "algorithmic_bytes": alg,
            "packed_us": round(t_packed, 3), "packed_GBs": round(alg / t_packed / 1e3, 1),
            "packed_frac": round(alg / t_packed / 1e3 / peak, 3), "packed_max_rel": packed_err,
            "packed_pdl_us": round(t_pdl, 3), "packed_pdl_GBs": round(alg / t_pdl / 1e3, 1),
            "packed_pdl_frac": round(alg / t_pdl / 1e3 / peak, 3),
            "regring_pdl_us": round(t_reg, 3), "regring_pdl_frac": round(alg / t_reg / 1e3 / peak, 3),
            "regring_max_rel": reg_err,
            "step_us": round(t_step, 3), "step_GBs": round(alg / t_step / 1e3, 1),
            "step_frac": round(alg / t_step / 1e3 / peak, 3), "step_max_rel": step_err,
            "ref_layout_us": round(t_ref, 3), "ref_layout_GBs": round(alg / t_ref / 1e3, 1),
            "ref_layout_max_rel": ref_err,
            "cublas_dense_us": round(t_dense, 3), "cublas_dense_GBs": round(dense_bytes / t_dense / 1e3, 1),
            "speedup_vs_cublas": round(t_dense / t_packed, 3),
            **tri,
        })
        print(json.dumps(rows[-1]), flush=True)
    return rows


def bench_rowwise(h: int, K: int, n: int, m: int, dev, reps: int, peak: float) -> dict:
    """Per-row N:M (BASELINE config 1 layout: values [w, h] + one uint8 offset
    per value) through nms_gemv_rowwise_f16; top-|w| packing of N(0, 0.02)."""
    from .nmsparse_linear import make_rowwise_topk

    lib = _lib.lib()
    w = K // m * n
    alg = h * w * 2 + h * w + K * 2 + h * 2
    nb = max(2, math.ceil(3 * L2_BYTES / alg) + 1)
    g = torch.Generator(device=dev).manual_seed(0)
    W0 = (torch.randn(h, K, device=dev, generator=g) * 0.02).to(torch.float16)
    md, mi = make_rowwise_topk(W0, n, m)
    del W0
    mats = [(md.clone(), mi.clone()) for _ in range(nb)]
    x = torch.randn(K, device=dev).to(torch.float16)
    outs = [torch.empty(h, device=dev, dtype=torch.float16) for _ in range(nb)]

    def fn(i):
        a, b = mats[i]
        return lambda s: _lib.check(lib.nms_gemv_rowwise_f16(x.data_ptr(), a.data_ptr(), b.data_ptr(),
                                                             outs[i].data_ptr(), K, w, h, n, m, s.cuda_stream),
                                    "nms_gemv_rowwise_f16")

    t = _graph_time_us([fn(i) for i in range(nb)], dev, reps)
    cols = (torch.arange(w, device=dev) // n)[:, None] * m + mi.long()
    ref = (md.float() * x.float()[cols]).sum(0)
    r = {"shape": f"{h}x{K}", "nm": f"{n}:{m} per-row", "algorithmic_bytes": alg,
         "rowwise_us": round(t, 3), "rowwise_GBs": round(alg / t / 1e3, 1), "rowwise_frac": round(alg / t / 1e3 / peak, 3),
         "rowwise_max_rel": _max_rel(outs[0], ref)}
    print(json.dumps(r), flush=True)
    del mats, outs
    torch.cuda.empty_cache()
    return r


def bench_dense_head(dev, reps: int, peak: float, V: int = 128256, K: int = 4096) -> dict:
    """The dense lm_head shape: cuBLAS torch.mv against this library's dense
    GEMV (the head launch of the decode step, without its argmax)."""
    lib = _lib.lib()
    x = torch.randn(K, device=dev).to(torch.float16)
    Wt = (torch.randn(V, K, device=dev) * 0.02).to(torch.float16)
    out = torch.empty(V, device=dev, dtype=torch.float16)
    by = V * K * 2 + K * 2 + V * 2
    t_cublas = _graph_time_us([lambda s: torch.mv(Wt, x, out=out)], dev, reps)
    a = _lib.NmsGemvFusedArgs()
    a.seg[0].packed = Wt.data_ptr()
    a.seg[0].rows = V
    a.nseg, a.flags = 1, _lib.NMS_FLAG_DENSE
    a.K = a.w = a.w_pad = K
    a.block_width = a.vec_width = 1
    a.x, a.out = x.data_ptr(), out.data_ptr()
    t_ours = _graph_time_us([lambda s: _lib.check(lib.nms_gemv_fused_f16(ctypes.byref(a), s.cuda_stream))], dev, reps)
    err = _max_rel(out, Wt.float() @ x.float())
    r = {"shape": f"{V}x{K}", "nm": "dense", "algorithmic_bytes": by,
         "packed_us": round(t_ours, 3), "packed_GBs": round(by / t_ours / 1e3, 1),
         "packed_frac": round(by / t_ours / 1e3 / peak, 3), "packed_max_rel": err,
         "cublas_dense_us": round(t_cublas, 3), "cublas_dense_GBs": round(by / t_cublas / 1e3, 1),
         "speedup_vs_cublas": round(t_cublas / t_ours, 3),
         "note": "1.05 GB per launch: far above L2, no rotation needed"}
    print(json.dumps(r), flush=True)
    return r


def bench_gemm(h: int, K: int, T: int, dev, reps: int, peak_gbs: float, peak_tf: float, M: int = 64) -> dict:
    """Prefill / batch > 1: gather + tcgen05 GEMM (nms_gemm_packed_f16) for T
    tokens against cuBLAS F.linear with a dense [h, K] fp16 weight.  Weight
    copies rotate over > 3x L2.  Roofline time = max(algorithmic bytes / HBM
    peak, sparse FLOPs (2 T h w) / tensor peak)."""
    lib = _lib.lib()
    packed, mi, w, nnz = make_sparse_device(K, h, M, 11, dev, std=0.02)
    w_pad = packed.shape[1]
    wbytes = packed.numel() * 2
    nb = max(2, math.ceil(3 * L2_BYTES / wbytes) + 1)
    packs = [packed] + [packed.clone() for _ in range(nb - 1)]
    x = torch.randn(T, K, device=dev).to(torch.float16)
    outs = [torch.empty(T, h, device=dev, dtype=torch.float16) for _ in range(nb)]
    n = ctypes.c_int64(0)
    _lib.check(lib.nms_gemm_workspace_bytes(T, w_pad, h, ctypes.byref(n)))
    ws = torch.empty(n.value, dtype=torch.uint8, device=dev)

    def ours(i):
        def f(s):
            _lib.check(lib.nms_gemm_packed_f16(x.data_ptr(), _lib.NMS_DTYPE_F16, packs[i].data_ptr(), mi.data_ptr(),
                                               outs[i].data_ptr(), T, K, w, w_pad, h, nnz, M, ws.data_ptr(),
                                               ws.numel(), s.cuda_stream), "nms_gemm_packed_f16")
        return f

    t_ours = _graph_time_us([ours(i) for i in range(nb)], dev, reps)
    ref = x.float() @ masked_dense(unpack(packed, w), mi, K, M).float().t()
    err = _max_rel(outs[0], ref)
    del ref
    dbytes = h * K * 2
    nd = max(2, math.ceil(3 * L2_BYTES / dbytes) + 1)
    Wd = [(torch.randn(h, K, device=dev) * 0.02).to(torch.float16) for _ in range(nd)]
    od = [torch.empty(T, h, device=dev, dtype=torch.float16) for _ in range(nd)]
    t_dense = _graph_time_us([(lambda i: lambda s: torch.matmul(x, Wd[i].t(), out=od[i]))(i) for i in range(nd)],
                             dev, reps)
    del Wd, od, packs
    by = wbytes + mi.numel() + T * K * 2 + T * h * 2
    flops = 2.0 * T * h * w
    t_roof = max(by / peak_gbs / 1e3, flops / peak_tf / 1e6)
    r = {"kind": "gemm", "shape": f"{h}x{K}", "nm": f"{nnz}:{M}", "T": T, "algorithmic_bytes": by,
         "sparse_flops": flops, "us": round(t_ours, 3), "GBs": round(by / t_ours / 1e3, 1),
         "TFLOPs": round(flops / t_ours / 1e6, 1), "roofline_us": round(t_roof, 3),
         "frac": round(t_roof / t_ours, 3), "bound": "hbm" if by / peak_gbs / 1e3 >= flops / peak_tf / 1e6 else "tensor",
         "max_rel": err, "cublas_dense_us": round(t_dense, 3),
         "cublas_dense_TFLOPs": round(2.0 * T * h * K / t_dense / 1e6, 1),
         "speedup_vs_cublas": round(t_dense / t_ours, 3)}
    print(json.dumps(r), flush=True)
    return r


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--shapes", default=",".join(f"{h}x{k}" for h, k in SHAPES))
    p.add_argument("--ratios", default=",".join(f"{n}:{m}" for n, m in RATIOS))
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--no-head", action="store_true")
    p.add_argument("--no-rowwise", action="store_true")
    p.add_argument("--triton-ref", action="store_true",
                   help="also time the reference's Triton kernel from baseline/_ref (a comparison arm)")
    p.add_argument("--out", default="", help="also write the rows as JSON to this file")
    p.add_argument("--gemm", default="", help="token counts for the prefill GEMM, e.g. 16,128,512,2048 "
                                              "(runs only the GEMM table)")
    args = p.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    peak, src = _peak_gbs()
    shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",") if s]
    ratios = [tuple(int(v) for v in r.split(":")) for r in args.ratios.split(",") if r]
    rows = []
    if args.gemm:
        tf, _ = _peak_tflops()
        for T in [int(v) for v in args.gemm.split(",") if v]:
            for h, K in shapes:
                rows.append(bench_gemm(h, K, T, dev, args.reps, peak, tf))
        print(json.dumps({"summary": True, "peak_GBs": peak, "peak_TFLOPs": tf, "peak_source": src,
                          "rows": len(rows)}), flush=True)
        return rows
    for h, K in shapes:
        rows += bench_shape(h, K, ratios, dev, args.reps, peak, triton_ref=args.triton_ref)
    if not args.no_rowwise:
        for h, K in shapes:
            rows.append(bench_rowwise(h, K, 32, 64, dev, args.reps, peak))
    if not args.no_head:
        rows.append(bench_dense_head(dev, args.reps, peak))
    print(json.dumps({"summary": True, "peak_GBs": peak, "peak_source": src, "rows": len(rows)}), flush=True)
    if args.out:
        Path(args.out).write_text(json.dumps({"peak_GBs": peak, "peak_source": src, "rows": rows}, indent=1))
    return rows


if __name__ == "__main__":
    main()
