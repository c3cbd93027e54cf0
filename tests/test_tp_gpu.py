"""Tensor-parallel decode on 2 GPUs (NCCL) against the single-GPU engine.

Two processes each build the same seeded model, shard it (tp.py) and decode
through their own CUDA graph -- with the plan executor and NCCL all-reduces,
and with the persistent step whose all-reduces run inside the kernel over
NVLink peer memory -- with the greedy-token all-gather captured; the
single-GPU engine on the unsharded model is the reference.  Tolerance: logits within 2e-2 x max|logit| (fp16
partial sums) and the same greedy tokens.  Skipped with fewer than 2 GPUs.
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


def _cfg():
    from spmv_decode_b200.model import ModelArgs

    return ModelArgs(block_size=128, vocab_size=2048, n_layer=2, n_head=8, n_local_heads=2, dim=1024,
                     intermediate_size=2048)


def _rank(rank, world, port, out, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    from spmv_decode_b200.generate import GraphDecoder
    from spmv_decode_b200.tp import build_tp_engine

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        eng, tp = build_tp_engine(_cfg(), (16, 32), world, rank, dev, max_seq=64, seed=5, history_len=64, mode=mode)
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


@pytest.mark.parametrize("mode", ["plan", "persistent"])
def test_tp2_engine_matches_single_gpu(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from spmv_decode_b200.engine import DecodeEngine
    from spmv_decode_b200.generate import GraphDecoder, build_model

    dev = torch.device("cuda:0")
    model = build_model(_cfg(), nm=(16, 32), device=dev, seed=5, init="device")
    eng = DecodeEngine(model, 64, history_len=64)
    ref_toks, ref_logits = GraphDecoder(eng).run(PROMPT, STEPS, keep_logits=True)
    ref_logits = ref_logits.cpu()
    eng.close()
    del eng, model
    torch.cuda.empty_cache()

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    toks, logits, dev_err = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    err = (logits.float() - ref_logits.float()).abs().amax(dim=1)
    scale = ref_logits.float().abs().amax(dim=1)
    assert bool((err <= TOL * scale).all()), (err / scale).max().item()
    assert toks == ref_toks
    assert dev_err == 0
