"""GPU: the verify forward (all kernels composed) against the torch fp32
restatement oracle/llama_ref.forward_full, and the speculative engine
end to end.

Tolerance (logits): max-abs <= 2e-2 relative to the logit scale
(max |ref| or 1), plus greedy-argmax agreement on rows whose fp32 top-2 margin
exceeds that tolerance (near-ties are reported, not asserted)."""
import pytest
import torch

from cudaforge_b200.model import TINY_DRAFT, TINY_TARGET, LlamaConfig, LlamaModel
from cudaforge_b200.runner import PagedRunner
from cudaforge_b200.speculative import SpeculativeEngine
from oracle import llama_ref

pytestmark = pytest.mark.gpu

SMALL_INT4 = LlamaConfig(2, 256, 4, 2, 64, 512, 1024)
SMALL_INT4_D128 = LlamaConfig(2, 512, 8, 2, 128, 768, 2048)


def _check_logits(ours, ref, tol=2e-2):
    ours = ours.float()
    scale = max(1.0, ref.abs().max().item())
    err = (ours - ref).abs().max().item() / scale
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > tol * scale
    agree = (ours.argmax(-1) == ref.argmax(-1))
    assert err <= tol, err
    assert agree[clear].all(), (agree[clear].float().mean().item())
    return err, agree.float().mean().item()


@pytest.mark.parametrize("cfg", [SMALL_INT4, SMALL_INT4_D128, TINY_TARGET], ids=["int4_d64", "int4_d128", "tiny_fp16"])
def test_verify_forward_matches_fp32_oracle(cfg):
    torch.manual_seed(0)
    model = LlamaModel(cfg, seed=0)
    B, S0, K = 3, 37, 4
    cache = model.make_cache(64)
    runner = PagedRunner(model, cache, seq_ids=[10, 11, 12])
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (B, S0), generator=g)
    runner.prefill(prompt[:, :-1].tolist())  # the last prompt token is the not-yet-cached row 0
    drafts = torch.randint(0, cfg.vocab, (B, K), generator=g)
    ids = torch.cat([prompt, drafts], 1).cuda()
    logits = runner.forward(ids)  # rows S0-1 .. S0+K-1  -> R = K + 1
    torch.cuda.synchronize()
    assert logits.shape == (B, K + 1, cfg.vocab)
    assert int(runner.status.item()) == 0
    ref = llama_ref.forward_full(model, ids)[:, -(K + 1):]
    _check_logits(logits, ref)


def test_prefill_then_commit_then_verify_chain():
    """Two verify steps with a per-sequence commit in between (ragged
    lengths): the committed K/V must serve the second step exactly as a full
    recompute would."""
    cfg = SMALL_INT4
    model = LlamaModel(cfg, seed=3)
    B, S0, K = 2, 20, 3
    runner = PagedRunner(model, model.make_cache(32), seq_ids=[0, 1])
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab, (B, S0), generator=g)
    runner.prefill(prompt[:, :-1].tolist())
    d1 = torch.randint(0, cfg.vocab, (B, K), generator=g)
    ids1 = torch.cat([prompt, d1], 1)
    runner.forward(ids1)
    runner.commit_upto([S0 - 1 + 2, S0 - 1 + 4])  # last emitted + 1 / + 3 drafts
    assert runner.committed == [S0 + 1, S0 + 3]
    seqs = [ids1[0, : S0 + 1].tolist() + [5], ids1[1, : S0 + 3].tolist() + [7]]
    lg = runner.forward(seqs)
    torch.cuda.synchronize()
    R = lg.shape[1]
    for b in range(B):
        ref = llama_ref.forward_full(model, torch.tensor([seqs[b]]).cuda())[0]
        _check_logits(lg[b], ref[-R:])


def test_speculative_step_greedy_matches_target_argmax():
    tgt = LlamaModel(TINY_TARGET, seed=0)
    drf = LlamaModel(TINY_DRAFT, seed=1)
    B, S0, K = 4, 24, 4
    seqs_ids = list(range(B))
    tr = PagedRunner(tgt, tgt.make_cache(64), seqs_ids)
    dr = PagedRunner(drf, drf.make_cache(64), seqs_ids)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, 32000, (B, S0), generator=g)
    tr.prefill(prompt[:, :-1].tolist())
    dr.prefill(prompt[:, :-1].tolist())
    eng = SpeculativeEngine(dr, tr, num_speculative_tokens=K, greedy=True)
    seqs = prompt.tolist()
    checked = 0
    for _ in range(3):
        res = eng.step(seqs)
        n = (res.per_sequence.num_accepted.cpu() + 1).tolist()
        for b in range(B):
            emitted = res.accepted_tokens[b, : n[b]].cpu().tolist()
            full = torch.tensor([seqs[b] + emitted]).cuda()
            ref = llama_ref.forward_full(tgt, full)[0]
            S = len(seqs[b])
            for j, tok in enumerate(emitted):
                row = ref[S - 1 + j]
                top2 = row.topk(2).values
                if (top2[0] - top2[1]).item() > 2e-2 * max(1.0, row.abs().max().item()):
                    assert tok == int(row.argmax()), (b, j)
                    checked += 1
            seqs[b] = seqs[b] + emitted
        assert tr.committed == [len(x) - 1 for x in seqs]
    assert checked > 0


@pytest.mark.parametrize("cfg,B", [(SMALL_INT4, 3), (LlamaConfig(1, 4096, 32, 8, 128, 14336, 4096), 64),
                                   (TINY_TARGET, 3)], ids=["int4_small", "int4_8b_layer_m384", "tiny_fp16"])
def test_fused_splitk_consumers_bit_identical(cfg, B):
    """The split-K reductions fused into RoPE / residual+RMSNorm / SwiGLU give the
    same bits as the reduction kernel followed by the plain ops."""
    from cudaforge_b200 import _lib
    model = LlamaModel(cfg, seed=4)
    S0, K = 29, 5
    runner = PagedRunner(model, model.make_cache(B * 4 + 8, max_batch=B), seq_ids=list(range(B)))
    g = torch.Generator().manual_seed(6)
    prompt = torch.randint(0, cfg.vocab, (B, S0), generator=g)
    runner.prefill(prompt[:, :-1].tolist())
    ids = torch.cat([prompt, torch.randint(0, cfg.vocab, (B, K), generator=g)], 1).cuda()
    M = B * (K + 1)
    from cudaforge_b200.gemm import MAX_FUSED_SPLITS
    sp = [_lib.lib().cf_gemm_splits(M, n, k, 0, int(cfg.quant == "int4")) for _, n, k in cfg.linear_shapes()]
    assert any(1 < x <= MAX_FUSED_SPLITS for x in sp), sp  # at least one fused split-K consumer runs
    outs = []
    for fuse in (False, True):
        model.fuse_splitk = fuse
        lg = runner.forward(ids).clone()
        bf = model.buffers(B, K + 1)
        outs.append((lg, bf["k_new"].clone(), bf["v_new"].clone()))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
