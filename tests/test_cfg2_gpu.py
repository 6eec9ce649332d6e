"""GPU: BASELINE config 2 -- speculative generation with the tiny fp16 pair
(target L4/d512/8x64/FFN1408, draft L1/d256/4x64/FFN704, V 32000), B=8,
128-token prompts, K=4, through the same code bench.py --config tiny times
(bench.generate_cfg2: paged prefill, device-resident draft loop, CUDA-graph
verify + accept + commit, draft advance).

  * logits: one verify step of the prefilled pair against the fp32
    restatement oracle/llama_ref.forward_rows over the same pools: max-abs
    <= 2e-2 of the logit scale, argmax agreement on rows with a clear top-2
    margin (agreement over all rows reported);
  * greedy generation: every emitted token equals the fp32 argmax of a full
    recompute of prompt + emitted prefix wherever the top-2 margin is clear;
  * T=0.8: every sequence reaches the requested length with in-range tokens."""
import pytest
import torch

import bench
from cudaforge_b200.model import TINY_DRAFT, TINY_TARGET
from oracle import llama_ref

pytestmark = pytest.mark.gpu

B, P, K = 8, 128, 4


def _prompts():
    return torch.randint(0, TINY_TARGET.vocab, (B, P), generator=torch.Generator().manual_seed(7))


def test_cfg2_verify_logits_vs_fp32():
    from cudaforge_b200.runner import PagedRunner
    from cudaforge_b200.model import LlamaModel
    from cudaforge_b200.verifier import BatchVerifier
    dev = torch.device("cuda")
    prompts = _prompts()
    target = LlamaModel(TINY_TARGET, device=dev, seed=1000)
    cache = target.make_cache(B * 16, max_batch=B, max_blocks_per_seq=16)
    ids = list(range(B))
    head = prompts[:, :-1].tolist()
    PagedRunner(target, cache, ids).prefill(head)
    ver = BatchVerifier(target, cache, ids, K, max_blocks_per_seq=16)
    ver.register_context(head, prompts[:, -1], registered=True)
    g = torch.Generator(device=dev).manual_seed(3)
    dt = torch.randint(0, TINY_TARGET.vocab, (B, K), generator=g, device=dev, dtype=torch.int32)
    dl = torch.randn(B, K, TINY_TARGET.vocab, generator=g, device=dev).to(TINY_TARGET.dtype)
    u = torch.rand(B, K + 1, generator=g, device=dev)
    tokens = torch.cat([ver.tokens[:, :1].clone(), dt], 1)
    ctx, tables = ver.ctx.clone(), ver.tables_dev.clone()
    ver.step(dt, dl, u)
    logits = target.buffers(B, K + 1)["logits"].view(B, K + 1, -1).float()
    cfg = cache.get_config()
    shp = (cfg.total_gpu_blocks, cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    ref = llama_ref.forward_rows(target, cache.key_pool.view(shp), cache.value_pool.view(shp), tables, ctx, tokens)
    scale = max(1.0, ref.abs().max().item())
    err = (logits - ref).abs().max().item() / scale
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > 2e-2 * scale
    agree = logits.argmax(-1) == ref.argmax(-1)
    print(f"cfg2 logits: max-abs/scale {err:.3e} (scale {scale:.3f}), argmax agreement "
          f"{agree.float().mean().item():.4f} of {agree.numel()} rows ({int(clear.sum())} with a clear margin)")
    assert err <= 2e-2
    assert agree[clear].all()


def test_cfg2_greedy_generation_follows_fp32_argmax():
    dev = torch.device("cuda")
    prompts = _prompts()
    out, ms, rounds, ver, target = bench.generate_cfg2(TINY_TARGET, TINY_DRAFT, prompts, K, 24, 1.0, True, dev)
    assert all(len(o) >= 24 for o in out)
    checked = agree = 0
    for b in range(B):
        full = torch.tensor([prompts[b].tolist() + out[b]], device=dev)
        ref = llama_ref.forward_full(target, full)[0]
        for j, tok in enumerate(out[b]):
            row = ref[P - 1 + j]
            top2 = row.topk(2).values
            if (top2[0] - top2[1]).item() > 2e-2 * max(1.0, row.abs().max().item()):
                checked += 1
                agree += int(tok == int(row.argmax()))
    print(f"cfg2 greedy: {agree}/{checked} emitted tokens with a clear fp32 margin equal the fp32 argmax; "
          f"{rounds} rounds, {sum(map(len, out)) / (rounds * B):.2f} tokens per sequence per round")
    assert checked > 0 and agree == checked


def test_cfg2_sampled_generation_runs_to_length():
    dev = torch.device("cuda")
    out, ms, rounds, _, _ = bench.generate_cfg2(TINY_TARGET, TINY_DRAFT, _prompts(), K, 32, 0.8, False, dev)
    assert all(len(o) >= 32 for o in out)
    assert all(0 <= t < TINY_TARGET.vocab for o in out for t in o)
