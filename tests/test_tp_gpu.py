"""Tensor-parallel decode on 2, 4 and 8 GPUs (NCCL) against the single-GPU engine.

World processes each build the same seeded model, shard it (tp.py) and decode
through their own CUDA graph -- with the plan executor and NCCL all-reduces,
and with the persistent step whose all-reduces run inside the kernel over
NVLink peer memory (plain peer loads and stores; no multicast) -- with the
greedy-token exchange captured; the single-GPU engine on the unsharded model
is the reference.  Models: a 2-layer toy, and 2 layers at the Llama-3.1-8B
(32:64) and Qwen3-32B (16:32, GQA 8, q/k-norm) widths of BASELINE configs 4
and 5.  Tolerance: logits within 2e-2 x max|logit| (fp16 partial sums) and
the same greedy tokens, except that a token may differ where the reference's
logit margin between the two tokens is within the measured logit error (an
fp16 near-tie that the order of the partial sums decides).  A case is
skipped when fewer GPUs than its world size are present.
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TOL = 2e-2
PROMPT = [11, 400, 7, 1999]
STEPS = 12


def _cfg(name="toy"):
    from spmv_decode_b200.model import ModelArgs

    if name == "toy":
        return ModelArgs(block_size=128, vocab_size=2048, n_layer=2, n_head=8, n_local_heads=2, dim=1024,
                         intermediate_size=2048)
    a = ModelArgs.from_name({"llama": "llama-3.1-8b", "qwen32": "qwen3-32b"}[name])
    a.n_layer = 2
    return a


NM = {"toy": (16, 32), "llama": (32, 64), "qwen32": (16, 32)}


def _rank(rank, world, port, out, mode, name="toy", temperature=0.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    from spmv_decode_b200.generate import GraphDecoder
    from spmv_decode_b200.tp import build_tp_engine

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        eng, tp = build_tp_engine(_cfg(name), NM[name], world, rank, dev, max_seq=64, seed=5, history_len=64,
                                  mode=mode, temperature=temperature, sample_seed=77)
        assert eng.mode == ("persistent_tp" if mode == "persistent" else "plan"), eng.mode
        gd = GraphDecoder(eng)
        toks, logits = gd.run(PROMPT, STEPS, keep_logits=True)
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits)
        full = torch.cat(parts, dim=1).cpu()
        del gd
        eng.close()
        tp.close()
        if rank == 0:
            out.put((toks, full, _lib_device_error()))
    finally:
        dist.destroy_process_group()


def _lib_device_error():
    from spmv_decode_b200 import _lib

    return _lib.device_error()


CASES = [
    (2, "toy", "plan"), (2, "toy", "persistent"),
    (2, "llama", "persistent"), (4, "llama", "persistent"), (8, "llama", "persistent"), (8, "llama", "plan"),
    (4, "qwen32", "persistent"), (8, "qwen32", "persistent"),
]


@pytest.mark.parametrize("world, name, mode", CASES, ids=[f"tp{w}-{n}-{m}" for w, n, m in CASES])
def test_tp_engine_matches_single_gpu(world, name, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.generate import GraphDecoder, build_model

    dev = torch.device("cuda:0")
    model = build_model(_cfg(name), nm=NM[name], device=dev, seed=5, init="device")
    eng = DecodeEngine(model, 64, history_len=64)
    ref_toks, ref_logits = GraphDecoder(eng).run(PROMPT, STEPS, keep_logits=True)
    ref_logits = ref_logits.float().cpu()
    eng.close()
    del eng, model
    torch.cuda.empty_cache()

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, mode, name)) for r in range(world)]
    for p in procs:
        p.start()
    toks, logits, dev_err = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dev_err == 0
    # The engines free-run: compare up to the first greedy token that
    # differs (if any), which must be an fp16 near-tie of the reference.
    first = len(PROMPT) - 1
    diverge = next((t for t, (a, b) in enumerate(zip(toks, ref_toks)) if a != b), None)
    rows = logits.shape[0] if diverge is None else first + diverge + 1
    logits = logits.float()[:rows]
    err = (logits - ref_logits[:rows]).abs().amax(dim=1)
    scale = ref_logits[:rows].abs().amax(dim=1)
    assert bool((err <= TOL * scale).all()), (err / scale).max().item()
    if diverge is not None:
        row = ref_logits[first + diverge]
        a, b = toks[diverge], ref_toks[diverge]
        assert (row[b] - row[a]).item() <= 2 * err[first + diverge].item(), (diverge, a, b)
    print(f"tp{world} {name} {mode}: worst rel logit err {(err / scale).max().item():.2e}, "
          f"tokens {'identical' if diverge is None else f'near-tie at step {diverge}'}")


def test_tp2_temperature_sampling_matches_single_gpu():
    """Sampling under tensor parallelism draws the single-GPU engine's tokens:
    the noise is keyed by the global vocabulary row, and the ranks exchange
    sampling keys instead of logits."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.generate import GraphDecoder, build_model

    dev = torch.device("cuda:0")
    model = build_model(_cfg("toy"), nm=NM["toy"], device=dev, seed=5, init="device")
    eng = DecodeEngine(model, 64, history_len=64, temperature=1.0, sample_seed=77)
    ref_toks, _ = GraphDecoder(eng).run(PROMPT, STEPS, keep_logits=True)
    eng.close()
    del eng, model
    torch.cuda.empty_cache()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, "persistent", "toy", 1.0)) for r in range(2)]
    for p in procs:
        p.start()
    toks, _, dev_err = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dev_err == 0
    assert toks == ref_toks
