"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference source tree is available (it imports the reference
from the directory named by the REFERENCE_ROOT environment variable, which
is required; GPU hosts do not have it):

    REFERENCE_ROOT=<path to the reference checkout> python tests/golden/make_golden.py

What it records, all produced by the reference's own code:
  packer.npz    -- _make_sparse (src/spmv/nmsparse_linear.py:14-33, shared-mask
                   branch, NM_KERNEL=triton_ptx): full arrays for small shapes,
                   SHA-256 of the bytes plus leading values for Llama shapes.
  packer_rowwise.npz -- _make_sparse's per-row branch (the layout of
                   NM_KERNEL=fp16 / fp16_split: mat_data [w, N] fp16 and
                   per-value offsets mat_index [w, N] uint8), same recording.
  gemv.npz      -- outputs of the reference Triton kernels
                   nmsparse_generic_kernel and nmsparse_a100_sm80_kernel
                   (triton_spmv.py:40-214), executed by the Triton interpreter
                   on the CPU.  The interpreter cannot run inline PTX, so
                   ptx_fma_f32 (triton_spmv.py:24-35, `fma.rn.f32`) is replaced
                   in memory by tl.fma, the same fused round-to-nearest fp32
                   multiply-add.  Launch parameters follow the wrapper
                   (triton_spmv.py:298-316) with one fixed autotune config.
  decode_*.npz  -- greedy decode with the reference decode path: gpt-fast
                   model.py Transformer (E2E_NO_FLASH=1 SDPA path) and HF
                   Qwen3ForCausalLM, linears replaced by the reference
                   swap_to_nmsparse, nmsparse::gemv executed by the
                   interpreted reference kernel.  Prompt tokens are fed one at
                   a time through the decode path (decode-only mode, as every
                   reference benchmark sets NM_DECODE_ONLY=1).
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
if "REFERENCE_ROOT" not in os.environ:
    raise SystemExit("set REFERENCE_ROOT to the reference checkout (the directory holding triton_spmv.py)")
REF = Path(os.environ["REFERENCE_ROOT"])

os.environ["TRITON_INTERPRET"] = "1"
os.environ["NM_KERNEL"] = "triton_ptx"
os.environ["NM_DECODE_ONLY"] = "1"
os.environ["E2E_NO_FLASH"] = "1"
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REF / "src" / "spmv"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

import nmsparse_linear as ref_linear  # noqa: E402  (reference src/spmv/nmsparse_linear.py)
import nmsparse_op as ref_op  # noqa: E402  (reference src/spmv/nmsparse_op.py)
import triton_spmv as ref_spmv  # noqa: E402  (reference triton_spmv.py)

assert Path(ref_linear.__file__).resolve().parent == (REF / "src" / "spmv").resolve(), ref_linear.__file__


@triton.jit
def _fma_rn_f32(x, y, acc):
    return tl.fma(x, y, acc)


ref_spmv.ptx_fma_f32 = _fma_rn_f32
for _k in (ref_spmv.nmsparse_generic_kernel, ref_spmv.nmsparse_a100_sm80_kernel):
    _k.fn.fn.__globals__["ptx_fma_f32"] = _fma_rn_f32


def run_ref_kernel(vec, mat_data, mat_index, w, h, nnz, m, variant="generic", block_rows=128, gpp=1):
    """The reference kernel on CPU tensors; returns the fp32 accumulator [1, h]."""
    num_groups = w // nnz
    out = torch.zeros((1, h), dtype=torch.float32)
    kern = ref_spmv.nmsparse_generic_kernel if variant == "generic" else ref_spmv.nmsparse_a100_sm80_kernel
    grid = (triton.cdiv(h, block_rows), triton.cdiv(num_groups, gpp))
    kern.fn[grid](
        vec, mat_data, mat_index, out, h, num_groups, vec.stride(1), mat_data.stride(0), mat_data.stride(1),
        NNZ=nnz, M=m, GROUPS_PER_PROGRAM=gpp, BLOCK_ROWS=block_rows,
    )
    return out


def cpu_gemv_op(x, mat_data, mat_index, w, h, block_width, vec_width):
    """CPU kernel for the reference nmsparse::gemv op: the triton_ptx branch of
    src/spmv/nmsparse_op.py:82-96 with the kernel launched directly (the
    wrapper's is_cuda checks are the only part bypassed)."""
    K = x.shape[-1]
    x2d = x.reshape(-1, K).contiguous()
    assert x2d.shape[0] == 1
    xh = x2d if x2d.dtype == torch.float16 else x2d.to(torch.float16)
    md = mat_data if mat_data.dtype == torch.float16 else mat_data.to(torch.float16)
    out = run_ref_kernel(xh, md, mat_index, int(w), int(h), int(block_width), int(vec_width))
    out = out.to(xh.dtype).to(x.dtype)
    return out.reshape(*x.shape[:-1], int(h))


ref_op.gemv.register_kernel("cpu")(cpu_gemv_op)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def make_packer():
    out = {}
    small = [(256, 128, 4, 0), (256, 128, 8, 1), (512, 256, 16, 2), (512, 128, 32, 3), (1024, 256, 64, 4),
             (1024, 128, 128, 5), (2048, 128, 256, 6)]
    for i, (K, N, M, seed) in enumerate(small):
        md, mi, w, nnz = ref_linear._make_sparse(K, N, M, seed, "cpu")
        out[f"small{i}_cfg"] = np.array([K, N, M, seed, w, nnz], dtype=np.int64)
        out[f"small{i}_mat_data"] = md.view(torch.int16).numpy()
        out[f"small{i}_mat_index"] = mi.numpy()
    big = [(4096, 4096, 64, 0), (4096, 6144, 64, 0), (14336, 4096, 64, 4), (4096, 14336, 16, 2),
           (4096, 4096, 4, 7), (4096, 4096, 256, 9)]
    for i, (K, N, M, seed) in enumerate(big):
        md, mi, w, nnz = ref_linear._make_sparse(K, N, M, seed, "cpu")
        out[f"big{i}_cfg"] = np.array([K, N, M, seed, w, nnz], dtype=np.int64)
        out[f"big{i}_sha_data"] = np.frombuffer(bytes.fromhex(sha(md.view(torch.int16))), dtype=np.uint8)
        out[f"big{i}_sha_index"] = np.frombuffer(bytes.fromhex(sha(mi)), dtype=np.uint8)
        out[f"big{i}_head_data"] = md[0, :16].view(torch.int16).numpy()
        out[f"big{i}_head_index"] = mi[:2].numpy()
    np.savez_compressed(HERE / "packer.npz", **out)
    print("packer.npz:", len(small), "small,", len(big), "big")


def make_packer_rowwise():
    """_make_sparse reads its mode from module globals at call time; switch
    them to what NM_KERNEL=fp16_split sets (src/spmv/nmsparse_linear.py:9-11)."""
    saved = (ref_linear._SHARED_MASK, ref_linear._FP16_SPARSE)
    ref_linear._SHARED_MASK, ref_linear._FP16_SPARSE = False, True
    try:
        out = {}
        small = [(256, 128, 4, 0), (512, 256, 16, 2), (1024, 128, 64, 4), (2048, 128, 256, 6)]
        for i, (K, N, M, seed) in enumerate(small):
            md, mi, w, nnz = ref_linear._make_sparse(K, N, M, seed, "cpu")
            assert md.dtype == torch.float16 and tuple(mi.shape) == (w, N)
            out[f"small{i}_cfg"] = np.array([K, N, M, seed, w, nnz], dtype=np.int64)
            out[f"small{i}_mat_data"] = md.view(torch.int16).numpy()
            out[f"small{i}_mat_index"] = mi.numpy()
        big = [(4096, 4096, 64, 0), (14336, 4096, 64, 4)]
        for i, (K, N, M, seed) in enumerate(big):
            md, mi, w, nnz = ref_linear._make_sparse(K, N, M, seed, "cpu")
            out[f"big{i}_cfg"] = np.array([K, N, M, seed, w, nnz], dtype=np.int64)
            out[f"big{i}_sha_data"] = np.frombuffer(bytes.fromhex(sha(md.view(torch.int16))), dtype=np.uint8)
            out[f"big{i}_sha_index"] = np.frombuffer(bytes.fromhex(sha(mi)), dtype=np.uint8)
        np.savez_compressed(HERE / "packer_rowwise.npz", **out)
        print("packer_rowwise.npz:", len(small), "small,", len(big), "big")
    finally:
        ref_linear._SHARED_MASK, ref_linear._FP16_SPARSE = saved


def make_gemv():
    out = {}
    cases = [(256, 128, 4, 11), (256, 256, 8, 12), (512, 128, 16, 13), (512, 256, 32, 14), (1024, 128, 64, 15),
             (1024, 256, 128, 16), (2048, 128, 256, 17), (768, 384, 32, 18)]
    for i, (K, N, M, seed) in enumerate(cases):
        md, mi, w, nnz = ref_linear._make_sparse(K, N, M, seed, "cpu")
        g = torch.Generator().manual_seed(1000 + seed)
        vec = torch.randn(1, K, generator=g, dtype=torch.float32).to(torch.float16)
        acc_generic = run_ref_kernel(vec, md, mi, w, N, nnz, M, "generic", block_rows=128, gpp=1)
        acc_a100 = run_ref_kernel(vec, md, mi, w, N, nnz, M, "a100", block_rows=64, gpp=2)
        op_out = torch.ops.nmsparse.gemv(vec.view(1, 1, K), md, mi, w, N, nnz, M)
        out[f"c{i}_cfg"] = np.array([K, N, M, seed, w, nnz], dtype=np.int64)
        out[f"c{i}_vec"] = vec.view(torch.int16).numpy()
        out[f"c{i}_mat_data"] = md.view(torch.int16).numpy()
        out[f"c{i}_mat_index"] = mi.numpy()
        out[f"c{i}_acc_generic"] = acc_generic.numpy()
        out[f"c{i}_acc_a100"] = acc_a100.numpy()
        out[f"c{i}_op_out"] = op_out.reshape(-1).view(torch.int16).numpy()
    np.savez_compressed(HERE / "gemv.npz", **out)
    print("gemv.npz:", len(cases), "cases")


def _greedy(logits: torch.Tensor) -> int:
    return int(torch.argmax(logits.reshape(-1)).item())


def make_decode_llama(steps=24, prompt_len=8):
    import model as ref_model  # reference model.py

    args = ref_model.ModelArgs(block_size=256, vocab_size=512, n_layer=2, n_head=2, dim=256,
                               intermediate_size=512, n_local_heads=1, rope_base=500000,
                               rope_scaling=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                                 original_max_position_embeddings=8192))
    torch.manual_seed(0)
    model = ref_model.Transformer(args)
    g = torch.Generator().manual_seed(77)
    with torch.no_grad():
        model.tok_embeddings.weight.copy_(torch.randn(args.vocab_size, args.dim, generator=g) * 0.02)
        model.output.weight.copy_(torch.randn(args.vocab_size, args.dim, generator=g) * 0.02)
    emb = model.tok_embeddings.weight.detach().to(torch.float16).clone()
    head = model.output.weight.detach().to(torch.float16).clone()
    model = model.to(torch.float16)
    M = 32
    cnt = ref_linear.swap_to_nmsparse(model, M, "cpu", seed=5)
    model.setup_caches(max_batch_size=1, max_seq_length=prompt_len + steps + 1)
    prompt = torch.randint(0, args.vocab_size, (prompt_len,), generator=torch.Generator().manual_seed(123))
    tokens, all_logits = [], []
    cur = int(prompt[0])
    with torch.no_grad():
        for pos in range(prompt_len + steps):
            idx = torch.tensor([[cur]], dtype=torch.int64)
            logits = model(None, idx, torch.tensor([pos], dtype=torch.int64))
            lg = logits[0, -1].to(torch.float16)
            all_logits.append(lg.view(torch.int16).numpy().copy())
            nxt = _greedy(lg)
            if pos + 1 < prompt_len:
                cur = int(prompt[pos + 1])
            else:
                tokens.append(nxt)
                cur = nxt
    np.savez_compressed(
        HERE / "decode_llama_tiny.npz",
        cfg=np.array([args.vocab_size, args.n_layer, args.n_head, args.n_local_heads, args.dim,
                      args.intermediate_size, M, 5, prompt_len, steps], dtype=np.int64),
        rope_base=np.array([args.rope_base], dtype=np.float64),
        emb=emb.view(torch.int16).numpy(), head=head.view(torch.int16).numpy(),
        prompt=prompt.numpy(), tokens=np.array(tokens, dtype=np.int64), logits=np.stack(all_logits),
        swapped=np.array([cnt], dtype=np.int64),
    )
    print("decode_llama_tiny.npz: swapped", cnt, "tokens", tokens[:8])


def make_decode_qwen3(steps=24, prompt_len=8):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.cache_utils import StaticCache

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                      rope_parameters={"rope_type": "default", "rope_theta": 1e6},
                      rms_norm_eps=1e-6, tie_word_embeddings=True, max_position_embeddings=256,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg)
    g = torch.Generator().manual_seed(78)
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * 0.02)
        for layer in model.model.layers:
            layer.self_attn.q_norm.weight.copy_(1.0 + 0.1 * torch.randn(cfg.head_dim, generator=g))
            layer.self_attn.k_norm.weight.copy_(1.0 + 0.1 * torch.randn(cfg.head_dim, generator=g))
            layer.input_layernorm.weight.copy_(1.0 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
            layer.post_attention_layernorm.weight.copy_(1.0 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
        model.model.norm.weight.copy_(1.0 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
    model = model.to(torch.float16).eval()
    M = 32
    cnt = ref_linear.swap_to_nmsparse(model.model, M, "cpu", seed=9)
    norms = {
        "q_norm": np.stack([l.self_attn.q_norm.weight.detach().view(torch.int16).numpy() for l in model.model.layers]),
        "k_norm": np.stack([l.self_attn.k_norm.weight.detach().view(torch.int16).numpy() for l in model.model.layers]),
        "in_norm": np.stack([l.input_layernorm.weight.detach().view(torch.int16).numpy() for l in model.model.layers]),
        "post_norm": np.stack([l.post_attention_layernorm.weight.detach().view(torch.int16).numpy()
                               for l in model.model.layers]),
        "final_norm": model.model.norm.weight.detach().view(torch.int16).numpy(),
    }
    emb = model.model.embed_tokens.weight.detach().view(torch.int16).numpy().copy()
    max_len = prompt_len + steps + 1
    try:
        cache = StaticCache(config=cfg, max_batch_size=1, max_cache_len=max_len, device="cpu", dtype=torch.float16)
    except TypeError:
        cache = StaticCache(config=cfg, max_cache_len=max_len)
    prompt = torch.randint(0, cfg.vocab_size, (prompt_len,), generator=torch.Generator().manual_seed(321))
    tokens, all_logits = [], []
    cur = int(prompt[0])
    with torch.no_grad():
        for pos in range(prompt_len + steps):
            out = model(input_ids=torch.tensor([[cur]]), position_ids=torch.tensor([[pos]]),
                        cache_position=torch.tensor([pos]), past_key_values=cache, use_cache=True,
                        attention_mask=torch.ones((1, pos + 1), dtype=torch.long))
            lg = out.logits[0, -1].to(torch.float16)
            all_logits.append(lg.view(torch.int16).numpy().copy())
            nxt = _greedy(lg)
            if pos + 1 < prompt_len:
                cur = int(prompt[pos + 1])
            else:
                tokens.append(nxt)
                cur = nxt
    np.savez_compressed(
        HERE / "decode_qwen3_tiny.npz",
        cfg=np.array([cfg.vocab_size, cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads,
                      cfg.hidden_size, cfg.intermediate_size, M, 9, prompt_len, steps], dtype=np.int64),
        rope_base=np.array([cfg.rope_parameters["rope_theta"]], dtype=np.float64), eps=np.array([cfg.rms_norm_eps]),
        emb=emb, prompt=prompt.numpy(), tokens=np.array(tokens, dtype=np.int64), logits=np.stack(all_logits),
        swapped=np.array([cnt], dtype=np.int64), **norms,
    )
    print("decode_qwen3_tiny.npz: swapped", cnt, "tokens", tokens[:8])


if __name__ == "__main__":
    which = sys.argv[1:] or ["packer", "rowwise", "gemv", "llama", "qwen3"]
    if "packer" in which:
        make_packer()
    if "rowwise" in which:
        make_packer_rowwise()
    if "gemv" in which:
        make_gemv()
    if "llama" in which:
        make_decode_llama()
    if "qwen3" in which:
        make_decode_qwen3()
