"""GPU: numerics of the benchmark configuration itself.

The Llama-3-8B-shaped W4A16 target (32 layers, d 4096, 32/8 heads, FFN
14336, V 128,256) verifies K=5 drafts for B=64 sequences with ~1,024-token
contexts through BatchVerifier in CUDA-graph mode -- the exact launch
sequence bench.py times (split-K plans of the M=384 GEMMs, the capture-time
max_context attention plan).  The step's logits are compared with the fp32
restatement oracle/llama_ref.forward_rows over the same paged pools:
max-abs error <= 2e-2 relative to the logit scale, and greedy-argmax
agreement on every row whose fp32 top-2 margin exceeds that tolerance.  The
graph step's acceptance decisions must equal the eager acceptance kernel's
on the same logits and uniforms, and those must equal the CPU oracle fed the
kernel's exported probabilities (bit-exact)."""
import numpy as np
import pytest
import torch

import oracle
from cudaforge_b200.accept import accept_sample
from cudaforge_b200.model import LLAMA_8B, LlamaModel
from cudaforge_b200.verifier import BatchVerifier
from oracle import llama_ref

pytestmark = pytest.mark.gpu


@pytest.mark.timeout(900)
def test_cfg3_graph_step_logits_and_acceptance():
    B, K, P = 64, 5, 1024
    R = K + 1
    dev = torch.device("cuda")
    model = LlamaModel(LLAMA_8B, device=dev, seed=1000)
    bps = (P + 8 * R) // 16 + 4
    cache = model.make_cache(B * bps + 8, max_batch=B, max_blocks_per_seq=bps + 4)
    ver = BatchVerifier(model, cache, list(range(B)), K, max_blocks_per_seq=bps + 4, use_graph=True)
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, LLAMA_8B.vocab, (B, P), generator=g)
    ver.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    gd = torch.Generator(device=dev).manual_seed(11)
    ver.fill_synthetic_kv(gd)
    V = LLAMA_8B.vocab
    dtok = torch.randint(0, V, (B, K), generator=gd, device=dev, dtype=torch.int32)
    dlog = (torch.randn(B, K, V, generator=gd, device=dev) * 2.0).to(torch.bfloat16)
    uni = torch.rand(3, B, R, generator=gd, device=dev)
    ver.step(dtok, dlog, uni[0])   # eager (counts the launches)
    assert ver.graphs is None
    # state the graph step starts from
    row0 = ver.tokens[:, 0].clone()
    ctx = ver.ctx.clone()
    tables = ver.tables_dev.clone()
    res = ver.step(dtok, dlog, uni[1])  # captures, then replays
    assert ver.graphs is not None
    logits = model.buffers(B, R)["logits"].view(B, R, V).clone()
    got_n, got_tok = res.num_accepted.clone(), res.tokens.clone()
    ver.check_status()

    tokens = torch.cat([row0.view(B, 1), dtok], 1)
    cfg = cache.get_config()
    shp = (cfg.total_gpu_blocks, cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    with torch.no_grad():
        ref = llama_ref.forward_rows(model, cache.key_pool.view(shp), cache.value_pool.view(shp), tables, ctx,
                                     tokens)
    scale = max(1.0, ref.abs().max().item())
    err = (logits.float() - ref).abs().max().item() / scale
    top2 = ref.topk(2, dim=-1).values
    margin = top2[..., 0] - top2[..., 1]
    clear = margin > 2e-2 * scale
    # rows whose fp32 top-2 margin exceeds twice the measured max error must agree
    decisive = margin > 2.0 * err * scale
    agree = logits.float().argmax(-1) == ref.argmax(-1)
    print(f"cfg3 logits: max-abs/scale {err:.3e} (scale {scale:.3f}); argmax agreement "
          f"{agree.float().mean().item():.4f} of {agree.numel()} rows, "
          f"{agree[decisive].float().mean().item() if decisive.any() else float('nan'):.4f} of "
          f"{int(decisive.sum())} rows with a top-2 margin > 2x the max error, {int(clear.sum())} rows with a "
          f"margin > the tolerance")
    assert err <= 2e-2, err
    assert agree[clear].all() and agree[decisive].all()

    # acceptance: graph step == eager kernel == oracle on the exported probabilities
    eager = accept_sample(dlog, logits, dtok, uni[1], export_probs=True)
    torch.cuda.synchronize()
    assert torch.equal(eager.num_accepted, got_n)
    na_e = eager.num_accepted.cpu().numpy()
    for b in range(B):
        assert torch.equal(eager.tokens[b, : na_e[b] + 1], got_tok[b, : na_e[b] + 1])
    tok, na, ef = oracle.accept(dtok.cpu().numpy(), eager.probs_draft.cpu().numpy(),
                                eager.probs_target.cpu().numpy(), uni[1].cpu().numpy(), -1)
    assert (na == na_e).all()
    for b in range(B):
        assert eager.emitted(b) == tok[b, : na[b] + 1].tolist()
