"""Benchmark: batch-1 decode ms/token under a CUDA graph (the reference's
headline metric), with the dominant kernel's achieved HBM bandwidth as its
roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model llama-3.1-8b] [--nm 32:64] [--ctx 512]

Protocol (reference: benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:145-189):
synthetic random-init weights, KV cache ~ N(0, 0.02) for CTX positions,
token 123 at position CTX, one decode step (embedding, all layers, output
head, greedy token) captured in a CUDA graph and replayed.  W untimed
replays, then K timed replays bracketed by a barrier and a device
synchronize, timed with CUDA events on the replay stream; every replay
streams all weights (> 8 GB), far more than the 126 MB L2, so no flush is
needed.  N > 1 runs tensor-parallel decode (one process per GPU, NCCL
all-reduce after the o- and down-projections); the time is the max over
ranks.

The JSON line also carries:
  e2e          the same metric through the public generation API with a
               pinned host->device token copy and a device->host read of the
               next token every step (positions advance);
  roofline     the dominant kernel of the timed region -- the persistent
               decode_step_kernel (one launch = one step): the step's
               algorithmic bytes / replay time vs the measured HBM copy
               bandwidth (MEASURED_PEAKS.json); gemv_roofline: the sparse
               GEMV kernel alone, timed live in a plan of the step's GEMVs;
  cpu_baseline the reference's torch CPU path (dense masked fp16 F.linear)
               on a bounded sample of the same workload, on this host;
  dense        the same engine with dense weights, and dense cuBLAS decode
               (torch modules with nn.Linear captured in a CUDA graph).
``--impl reference`` prints the CPU reference arm's line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "decode ms/token bs=1 (CUDA graph)"
UNIT = "ms/token"
# Published reference number for this exact metric and configuration:
# Llama 3.1 8B, 32:64, CTX=512, fixed-context CUDA-graph decode, A100-SXM4-80GB
# (reference README.md:93).
PUBLISHED = {("llama-3.1-8b", "32:64"): (6.8521, "A100-SXM4-80GB", "README.md:93"),
             ("qwen3-32b", "16:32"): (33.7054, "A100-SXM4-80GB", "README.md:118")}


def env_defaults() -> dict:
    """Defaults from the reference benchmark's environment (benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:97-105):
    NM_M (0 = dense, else M with N = M/2), CTX, BENCH_WARMUP, and BENCH_REPEAT x BENCH_INNER timed
    replays.  Only variables that are set apply; explicit flags override them."""
    env = os.environ
    d = {"ctx": int(env.get("CTX", 512))}
    if "NM_M" in env:
        m = int(env["NM_M"])
        if m not in (0, 4, 8, 16, 32, 64, 128, 256):
            raise ValueError("Unsupported NM_M")
        d["nm"] = "dense" if m == 0 else f"{m // 2}:{m}"
    if "BENCH_WARMUP" in env:
        d["warmup"] = int(env["BENCH_WARMUP"])
    if "BENCH_REPEAT" in env or "BENCH_INNER" in env:
        d["inner"] = int(env.get("BENCH_INNER", "10"))
        d["steps"] = int(env.get("BENCH_REPEAT", "30")) * d["inner"]
    if min(d["ctx"], d.get("warmup", 1), d.get("steps", 1)) < 1:
        raise ValueError("CTX, warmup, repeat, inner must be positive")
    return d


def parse_args():
    env = env_defaults()
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=env.get("steps", 1000))
    p.add_argument("--warmup", type=int, default=env.get("warmup", 50))
    p.add_argument("--inner", type=int, default=env.get("inner", 10),
                   help="replays per timed sample (the reference's BENCH_INNER); samples = steps // inner")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="llama-3.1-8b")
    p.add_argument("--nm", default=env.get("nm", "32:64"), help="N:M pattern, or 'dense'")
    p.add_argument("--ctx", type=int, default=env["ctx"])
    p.add_argument("--e2e-steps", type=int, default=256)
    p.add_argument("--prefetch", type=int, default=0, help="per-warp L2 look-ahead bytes inside a GEMV")
    p.add_argument("--next-prefetch", type=int, default=0,
                   help="bytes of the following GEMV's weights prefetched into L2 by each launch")
    p.add_argument("--no-dense", action="store_true", help="skip the dense controls")
    p.add_argument("--no-compile", action="store_true", help="skip the torch.compile dense control")
    p.add_argument("--no-sampled", action="store_true", help="skip the temperature-1.0 sampled-step timing")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--cpu-layers", type=int, default=2)
    p.add_argument("--mode", choices=["auto", "persistent", "plan"], default="auto",
                   help="decode-step executor: one persistent kernel or a per-kernel launch plan")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--layers", type=int, default=0,
                   help="profiling only: keep the model's shapes but this many decoder layers")
    p.add_argument("--vocab", type=int, default=0, help="profiling only: override the vocabulary size")
    p.add_argument("--sub-model", default="qwen3-32b:16:32",
                   help="second workload timed in the same run at the same N (BASELINE config 5, the "
                        "tensor-parallel model), as model:n:m; 'none' skips it")
    p.add_argument("--sub-steps", type=int, default=200)
    return p.parse_args()


def model_config(args):
    """The named configuration, with the profiling-only layer / vocabulary
    overrides applied."""
    import dataclasses

    from spmv_decode_b200.model import ModelArgs

    cfg = ModelArgs.from_name(args.model)
    over = {}
    if args.layers:
        over["n_layer"] = args.layers
    if args.vocab:
        over["vocab_size"] = args.vocab
    return dataclasses.replace(cfg, **over) if over else cfg


def workload_name(args) -> str:
    w = f"{args.model}-arch {args.nm} decode, ctx {args.ctx}, batch 1"
    if args.layers or args.vocab:
        w += f" [profiling case: {args.layers or 'all'} layers, vocab {args.vocab or 'full'}]"
    return w


def measured_peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` on `workload` from the committed ncu
    summary (profiles/traffic.json), if any."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    d = json.loads(f.read_text())
    return d.get(kernel, {}).get(workload)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def time_graph(graph, stream, steps: int, warmup: int, world: int, inner: int = 0) -> float:
    """Mean ms per replay over ``steps`` timed replays; max over ranks.
    ``stream`` must be the current stream (the one replay() launches on).
    See time_graph_stats for the per-sample statistics."""
    return time_graph_stats(graph, stream, steps, warmup, world, inner)["mean"]


def time_graph_stats(graph, stream, steps: int, warmup: int, world: int, inner: int = 0) -> dict:
    """Time ``steps`` replays as ``steps // inner`` samples of ``inner``
    replays each (the reference's BENCH_REPEAT x BENCH_INNER,
    benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:183-189): CUDA events
    between samples on the replay stream, one device synchronize before and
    after the whole timed region.  Returns the median, mean and stdev of the
    per-sample ms per replay (the mean is over all replays); under
    torchrun each is the max over ranks."""
    assert stream == torch.cuda.current_stream(), "time on the stream the graph replays on"
    inner = max(1, min(inner or min(10, steps), steps))
    reps = max(1, steps // inner)
    steps = reps * inner
    for _ in range(warmup):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    ev[0].record(stream)
    for r in range(reps):
        for _ in range(inner):
            graph.replay()
        ev[r + 1].record(stream)
    torch.cuda.synchronize()
    samples = [ev[r].elapsed_time(ev[r + 1]) / inner for r in range(reps)]
    out = {"median": statistics.median(samples), "mean": ev[0].elapsed_time(ev[-1]) / steps,
           "stdev": statistics.pstdev(samples) if reps > 1 else 0.0, "repeat": reps, "inner": inner,
           "steps": steps}
    if world > 1:
        dist.barrier()
        t = torch.tensor([out["median"], out["mean"], out["stdev"]], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out["median"], out["mean"], out["stdev"] = (float(v) for v in t.tolist())
    return out


def sub_record(args, world: int, rank: int, dev, peaks: dict) -> dict:
    """ms/token of a second model at the same GPU count (tensor parallel over
    the ranks for N > 1): BASELINE config 5, Qwen3-32B architecture 16:32 by
    default, fixed-context CUDA-graph decode at the same CTX, max over ranks;
    with its weight-bytes roofline per GPU."""
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.generate import build_model
    from spmv_decode_b200.model import ModelArgs

    name, n, m = args.sub_model.split(":")
    nm = (int(n), int(m))
    cfg = ModelArgs.from_name(name)
    max_seq = args.ctx + 8
    t0 = time.time()
    if world > 1:
        from spmv_decode_b200.tp import build_tp_engine

        eng, tp = build_tp_engine(cfg, nm, world, rank, dev, max_seq=max_seq, seed=args.seed, history_len=8,
                                  mode=args.mode)
    else:
        tp = None
        model = build_model(cfg, nm=nm, device=dev, seed=args.seed, init="device")
        eng = DecodeEngine(model, max_seq, history_len=8, mode=args.mode)
    build_s = time.time() - t0
    eng.fill_synthetic_cache(args.ctx, seed=args.seed)
    eng.token_in.fill_(123)
    graph = eng.capture(advance=False)
    stream = torch.cuda.current_stream(dev)
    st = time_graph_stats(graph, stream, args.sub_steps, 10, world, args.inner)
    sb = eng.step_bytes(args.ctx)
    if world > 1:
        t = torch.tensor([float(sb["total"])], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per_gpu = float(t.item())
    else:
        per_gpu = float(sb["total"])
    ideal = per_gpu / peaks["hbm_gbs"] / 1e6
    out = {"workload": f"{name}-arch {n}:{m} decode, ctx {args.ctx}, batch 1", "parallelism": f"tp{world}",
           "executor": eng.mode, "ms_per_token": round(st["median"], 4), "mean_ms": round(st["mean"], 4),
           "steps": st["steps"], "bytes_per_gpu_per_token": int(per_gpu), "ideal_ms": round(ideal, 4),
           "frac_of_hbm_roofline": round(ideal / st["median"], 4), "build_s": round(build_s, 1),
           "note": "max over ranks; weight-bytes roofline of the busiest GPU at the measured HBM bandwidth"}
    pub = PUBLISHED.get((name, f"{n}:{m}"))
    if pub is not None:
        out["published_reference"] = {"value": pub[0], "hardware": pub[1], "source": pub[2]}
    del graph
    eng.close()
    if tp is not None:
        if world > 1:
            dist.barrier()
        tp.close()
    del eng
    torch.cuda.empty_cache()
    return out


def run_reference_arm(args, world: int, rank: int) -> None:
    """The reference's own CPU implementation of the path (torch CPU F.linear
    on dense masked fp16 weights), timed on this host's cores."""
    if rank != 0:
        return
    from oracle.decode_oracle import cpu_decode_sample
    from spmv_decode_b200.model import ModelArgs

    cfg = model_config(args)
    nm = None if args.nm == "dense" else tuple(int(v) for v in args.nm.split(":"))
    threads = os.cpu_count() or 1
    # Each "step" is one sampled token; keep the run bounded.
    steps = max(1, min(args.steps, 5))
    warm = max(3, min(args.warmup, 5))
    r = cpu_decode_sample(cfg, nm, args.ctx, sample_layers=args.cpu_layers, steps=steps, threads=threads,
                          seed=args.seed, warmup=warm)
    v = r["ms_per_token"]
    line = {
        "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": round(v, 3), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 (torch CPU F.linear)", "data": "synthetic random-init weights",
        "impl": "reference",
        "config": {"workload": workload_name(args),
                   "model": args.model, "nm": args.nm, "ctx": args.ctx, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": r["threads"], "kind": "port",
                         "sample": r["sample"]},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


_JSON_FD = None


def emit(line: dict) -> None:
    """The one JSON line on the process's original stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def result_line(ctx: int, nm: str, mode: str, warmup: int, st: dict) -> str:
    """The reference benchmark's summary line (benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:186-189),
    the one its runner scripts parse (scripts/run_bench_qwen_32b_fp16.sh:215-219): the median,
    mean and stdev over ``repeat`` samples of ``inner`` replays each."""
    if nm == "dense":
        tag = "dense_float16"
    else:
        n, m = nm.split(":")
        tag = f"M={m}({n}:{m})"
    return (f"RESULT CTX={ctx} {tag} dtype=float16 actual_mode=b200_{mode} "
            f"measurement=fixed_context_cuda_graph warmup={warmup} repeat={st['repeat']} "
            f"decode_ms_per_token={st['median']:.6f} mean={st['mean']:.6f} stdev={st['stdev']:.6f}")


def check_import_origin() -> None:
    """Time only this tree: the package and its native library must come from
    the directory bench.py sits in, not a stray installed copy (the reference's
    "Foreign import" guard, benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:91-94)."""
    import spmv_decode_b200
    from spmv_decode_b200 import _lib

    pkg = Path(spmv_decode_b200.__file__).resolve().parent
    for path in (pkg, Path(_lib.LIB_PATH).resolve()):
        if ROOT not in path.parents:
            raise RuntimeError(f"Foreign import: {path} is outside {ROOT}")
    # ... and the library must have been built from the sources beside it.
    from spmv_decode_b200 import build as _build

    if _lib.source_hash() != _build.source_hash():
        raise RuntimeError(f"stale library {_lib.LIB_PATH}: built from sources {_lib.source_hash()}, the tree has "
                           f"{_build.source_hash()}; rebuild with `python -m spmv_decode_b200.build`")


def main():
    global _JSON_FD
    args = parse_args()
    check_import_origin()
    # Libraries (NCCL's version banner, warnings) may write to file
    # descriptor 1: send it to stderr so stdout carries only the JSON line.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world == 1 and args.gpus > 1:
        raise SystemExit("for --gpus > 1 launch with torch.distributed.run (one process per GPU)")
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return

    from spmv_decode_b200 import _lib
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.generate import build_model
    from spmv_decode_b200.model import ModelArgs

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    nm = None if args.nm == "dense" else tuple(int(v) for v in args.nm.split(":"))
    cfg = model_config(args)
    max_seq = args.ctx + 1 + args.e2e_steps + 8
    t_build = time.time()
    tp = None
    if world > 1:
        from spmv_decode_b200.tp import build_tp_engine

        eng, tp = build_tp_engine(cfg, nm, world, rank, dev, max_seq=max_seq, seed=args.seed,
                                  prefetch_bytes=args.prefetch, next_prefetch_bytes=args.next_prefetch,
                                  history_len=max_seq, mode=args.mode)
    else:
        model = build_model(cfg, nm=nm, device=dev, seed=args.seed, init="device")
        eng = DecodeEngine(model, max_seq, prefetch_bytes=args.prefetch, next_prefetch_bytes=args.next_prefetch,
                           history_len=max_seq, mode=args.mode)
    build_s = time.time() - t_build

    # ---- headline: fixed-context graph replay --------------------------------
    eng.fill_synthetic_cache(args.ctx, seed=args.seed)
    eng.token_in.fill_(123)
    graph = eng.capture(advance=False)
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(local_rank)
    st = time_graph_stats(graph, stream, args.steps, args.warmup, world, args.inner)
    ms = st["median"]
    clk = clocks.stop()
    assert torch.isfinite(eng.logits.float()).all(), "non-finite logits after replay"
    # Kernels of this library per step: one persistent kernel, or the plan's
    # launches (the plan holds the head twice: fixed and advancing variants).
    launches_per_step = {"persistent": 1, "persistent_tp": 1}.get(eng.mode, eng.size() - 1)
    engine_mode = eng.mode
    dev_err = _lib.device_error()

    # ---- e2e: public generation API with host I/O every step ------------------
    from spmv_decode_b200.generate import GraphDecoder

    gd = GraphDecoder(eng)
    e2e_steps = min(args.e2e_steps, max_seq - args.ctx - 2)
    tok_host = torch.tensor([123], dtype=torch.int64).pin_memory()
    out_host = torch.zeros(1, dtype=torch.int64).pin_memory()
    eng.pos.fill_(args.ctx)
    for _ in range(3):
        eng.token_in.copy_(tok_host, non_blocking=True)
        gd.replay()
        out_host.copy_(eng.token_out, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    eng.pos.fill_(args.ctx)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        eng.token_in.copy_(tok_host, non_blocking=True)
        gd.replay()
        out_host.copy_(eng.token_out, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        tok_host[0] = out_host[0]
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # ---- the reference's timed work includes sampling: the same step with ----
    # ---- temperature 1.0 (generate.py:46-63, top_k None as in its bench) ----
    sampled = None
    if world == 1 and not args.no_sampled:
        seng = DecodeEngine(model, max_seq, history_len=8, mode=args.mode, temperature=1.0, sample_seed=args.seed)
        seng.fill_synthetic_cache(args.ctx, seed=args.seed)
        seng.token_in.fill_(123)
        sg_ = seng.capture(advance=False)
        sst = time_graph_stats(sg_, stream, max(20, args.steps // 4), 10, world, args.inner)
        sampled = {"temperature": 1.0, "top_k": None, "ms_per_token": round(sst["median"], 4),
                   "note": "same step, token sampled from softmax(logits) in the head kernel (Gumbel-max with "
                           "Philox4x32-10 noise), as the reference's timed decode samples"}
        del sg_
        seng.close()
        del seng

    # ---- roofline: the sparse GEMV kernel timed live --------------------------
    plan, gemv_bytes = eng.gemv_plan()
    n_gemv = sum(1 for r in eng.gemv_records if not r["argmax"])

    s2 = torch.cuda.Stream(dev)
    s2.wait_stream(stream)
    with torch.cuda.stream(s2):
        for _ in range(3):
            _lib.check(_lib.lib().nms_plan_launch(plan, 0, n_gemv, s2.cuda_stream))
    stream.wait_stream(s2)
    torch.cuda.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=s2):
        _lib.check(_lib.lib().nms_plan_launch(plan, 0, n_gemv, s2.cuda_stream))
    gemv_ms = time_graph(g2, stream, max(10, args.steps // 4), 5, world)
    _lib.lib().nms_plan_destroy(plan)
    peaks = measured_peaks()
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    workload = workload_name(args)
    # The plan's GEMV launches run the shared-memory ring kernel unless the
    # L2 look-ahead option sends them to the register-ring kernel.
    gemv_kernel = "gemv_packed_kernel" if args.prefetch > 0 else "gemv_ring_kernel"
    gemv_roofline = {"bound": "hbm", "kernel": gemv_kernel, "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": profiled_traffic(gemv_kernel, workload),
                     "algorithmic_bytes": gemv_bytes, "launches": n_gemv,
                     "mean_launch_us": round(gemv_ms * 1e3 / n_gemv, 3),
                     "note": "the step's GEMV launches alone (plan executor), timed in their own CUDA graph"}
    sb = eng.step_bytes(args.ctx)
    # The dominant kernel of the timed region: with the persistent executor
    # the whole step is one decode_step_kernel launch, so its duration is the
    # replay time; with the plan executor the GEMV kernel above dominates.
    if engine_mode in ("persistent", "persistent_tp"):
        step_achieved = sb["total"] / (ms * 1e-3) / 1e9
        kname = "decode_step_kernel"
        roofline = {"bound": "hbm", "kernel": kname, "achieved": round(step_achieved, 1),
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(step_achieved / peaks["hbm_gbs"], 4),
                    "peak_source": peaks["source"],
                    "traffic": profiled_traffic("decode_step_kernel", workload) if world == 1 else None,
                    "algorithmic_bytes": sb["total"], "launches": 1, "mean_launch_us": round(ms * 1e3, 3)}
    else:
        roofline = dict(gemv_roofline)
        roofline.pop("note")
    step_roofline = {"bytes_per_token": sb, "ideal_ms": round(sb["total"] / peaks["hbm_gbs"] / 1e6, 4),
                     "frac": round(sb["total"] / peaks["hbm_gbs"] / 1e6 / ms, 4)}
    del g2, graph, gd
    eng.close()
    del eng
    if world == 1:
        del model
    torch.cuda.empty_cache()

    # ---- second workload at the same N (the tensor-parallel model) -----------
    sub = None
    if args.sub_model != "none" and not args.layers and not args.vocab:
        sub = sub_record(args, world, rank, dev, peaks)

    # ---- dense controls ------------------------------------------------------
    dense = None
    if not args.no_dense and nm is not None and world == 1:
        dense = {}
        dmodel = build_model(cfg, nm=None, device=dev, seed=args.seed + 1, init="device")
        # Our engine with dense weights on each executor ("auto" times both
        # and keeps the faster, so the control is not held to one executor).
        dmodes = ["persistent", "plan"] if args.mode == "auto" else [args.mode]
        for dmode in dmodes:
            deng = DecodeEngine(dmodel, args.ctx + 8, prefetch_bytes=args.prefetch,
                                next_prefetch_bytes=args.next_prefetch, mode=dmode)
            deng.fill_synthetic_cache(args.ctx, seed=args.seed)
            deng.token_in.fill_(123)
            dg = deng.capture(advance=False)
            dense[f"engine_dense_{deng.mode}_ms"] = round(time_graph(dg, stream, max(20, args.steps // 4), 10,
                                                                     world), 4)
            del dg
            deng.close()
            del deng
            torch.cuda.empty_cache()
        dense["engine_dense_ms"] = min(v for k, v in dense.items() if k.startswith("engine_dense_"))
        # cuBLAS: the torch module path (nn.Linear -> cuBLAS, SDPA attention)
        # captured in a CUDA graph, like the reference's dense baseline.
        dmodel.setup_caches(1, args.ctx + 8)
        for blk in dmodel.layers:
            blk.attn.kv_cache.k_cache.normal_(std=0.02)
            blk.attn.kv_cache.v_cache.normal_(std=0.02)
        idx = torch.tensor([[123]], device=dev)
        ipos = torch.tensor([args.ctx], device=dev)
        with torch.inference_mode():
            s3 = torch.cuda.Stream(dev)
            s3.wait_stream(stream)
            with torch.cuda.stream(s3):
                for _ in range(3):
                    torch.argmax(dmodel(None, idx, ipos)[0, -1])
            stream.wait_stream(s3)
            torch.cuda.synchronize()
            g3 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g3, stream=s3):
                torch.argmax(dmodel(None, idx, ipos)[0, -1])
            dense["cublas_graph_ms"] = round(time_graph(g3, stream, max(20, args.steps // 4), 10, world), 4)
            del g3
            # The reference's dense protocol: torch.compile(decode_one_token,
            # mode="default"), then CUDA-graph capture of the compiled step
            # (benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:155-170).
            if not args.no_compile:
                t_c = time.time()
                try:
                    step = torch.compile(lambda i, p: torch.argmax(dmodel(None, i, p)[0, -1]), mode="default")
                    with torch.cuda.stream(s3):
                        for _ in range(3):
                            step(idx, ipos)
                    stream.wait_stream(s3)
                    torch.cuda.synchronize()
                    g4 = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g4, stream=s3):
                        step(idx, ipos)
                    dense["torch_compile_graph_ms"] = round(
                        time_graph(g4, stream, max(20, args.steps // 4), 10, world), 4)
                    del g4
                except Exception as exc:  # the control is reported, not required
                    dense["torch_compile_graph_ms"] = None
                    dense["torch_compile_error"] = f"{type(exc).__name__}: {str(exc)[:200]}"
                dense["torch_compile_s"] = round(time.time() - t_c, 1)
        del dmodel
        torch.cuda.empty_cache()
        dense["speedup_vs_engine_dense"] = round(dense["engine_dense_ms"] / ms, 3)
        dense["speedup_vs_cublas"] = round(dense["cublas_graph_ms"] / ms, 3)
        candidates = {k: dense.get(k) for k in ("engine_dense_ms", "cublas_graph_ms", "torch_compile_graph_ms")}
        best_k = min((k for k, v in candidates.items() if v), key=lambda k: candidates[k])
        dense["best_dense"] = best_k
        dense["speedup_vs_best_dense"] = round(candidates[best_k] / ms, 3)

    # ---- CPU baseline (rank 0, N=1) -----------------------------------------
    cpu = None
    if not args.no_cpu and world == 1 and rank == 0:
        from oracle.decode_oracle import cpu_decode_sample

        r = cpu_decode_sample(cfg, nm, args.ctx, sample_layers=args.cpu_layers, steps=3,
                              threads=os.cpu_count(), seed=args.seed, warmup=3, single_thread_steps=1)
        cpu = {"value": round(r["ms_per_token"], 3), "unit": UNIT, "cores": r["threads"], "kind": "port",
               "sample": r["sample"],
               # the same sample on one host thread (torch.set_num_threads(1)), one timed step
               "single_thread": {"value": round(r["single_thread_ms_per_token"], 3), "unit": UNIT, "cores": 1}}

    if rank == 0:
        pub = PUBLISHED.get((args.model, args.nm))
        line = {
            "metric": METRIC, "value": round(ms, 4), "unit": UNIT, "n_gpus": world, "steps": st["steps"],
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
            "samples": {"repeat": st["repeat"], "inner": st["inner"], "median_ms": round(st["median"], 4),
                        "mean_ms": round(st["mean"], 4), "stdev_ms": round(st["stdev"], 5),
                        "note": "value = median of the samples (the reference's decode_ms_per_token)"},
            "vs_baseline": None if (pub is None or args.layers or args.vocab) else round(ms / pub[0], 4),
            "dtype": "f16 (fp32 accumulate)",
            "data": "synthetic: random-init weights N(0,0.02), KV cache N(0,0.02) (reference fixed-context protocol)",
            "config": {"workload": workload, "model": args.model, "nm": args.nm, "ctx": args.ctx,
                       "parallelism": f"tp{world}", "prefetch": args.prefetch, "next_prefetch": args.next_prefetch,
                       "executor": engine_mode,
                       "l2": "no flush: every replay streams all weights (>> 126 MB L2)"},
            "e2e": {"value": round(e2e_ms, 4), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                    "steps": e2e_steps, "note": "public generation API, host token in/out every step"},
            "roofline": roofline,
            "gemv_roofline": gemv_roofline,
            "step_roofline": step_roofline,
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_step * st["steps"],
            "clocks": clk,
            "dense": dense,
            "sub": sub,
            "sampled": sampled,
            "baseline_published": None if pub is None else {"value": pub[0], "hardware": pub[1], "source": pub[2]},
            "build_s": round(build_s, 1),
            "device_error": dev_err,
        }
        emit(line)
        # stdout carries only the JSON line; the reference's RESULT line goes to stderr.
        print(result_line(args.ctx, args.nm, engine_mode, args.warmup, st), file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
        tp.close()
        del tp
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
