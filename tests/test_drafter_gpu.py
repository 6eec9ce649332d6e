"""GPU: the device-resident draft loop (BatchDrafter) against the torch fp32
restatement oracle/llama_ref.forward_full.

Each round's K draft-logit rows must match a full fp32 recompute of the
sequence plus the drafts (max-abs <= 2e-2 of the logit scale, greedy argmax
agreement on rows with a clear top-2 margin); acceptance outcomes are
simulated between rounds, including all K accepted (the next round's step 0
then covers the draft the model never saw) and none accepted."""
import pytest
import torch

from cudaforge_b200.accept import AcceptResult, accept_sample
from cudaforge_b200.drafter import BatchDrafter
from cudaforge_b200.model import TINY_DRAFT, LlamaConfig, LlamaModel
from cudaforge_b200.runner import PagedRunner
from oracle import llama_ref

pytestmark = pytest.mark.gpu

SMALL_INT4 = LlamaConfig(2, 256, 4, 2, 64, 512, 1024)


def _check_logits(ours, ref, tol=2e-2):
    ours = ours.float()
    scale = max(1.0, ref.abs().max().item())
    assert (ours - ref).abs().max().item() / scale <= tol
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > tol * scale
    assert (ours.argmax(-1) == ref.argmax(-1))[clear].all()
    return clear


def _setup(cfg, B, S0, K, seed, use_graph=False, greedy=True, temperature=1.0):
    model = LlamaModel(cfg, seed=seed)
    cache = model.make_cache(B * 8 + 16, max_blocks_per_seq=16)
    g = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(0, cfg.vocab, (B, S0), generator=g)
    runner = PagedRunner(model, cache, list(range(B)))
    runner.prefill(prompt[:, :-1].tolist())
    dr = BatchDrafter(model, cache, list(range(B)), K, greedy=greedy, temperature=temperature,
                      max_blocks_per_seq=16, use_graph=use_graph)
    dr.register_context(prompt[:, :-1].tolist(), prompt[:, -1], registered=True)
    return model, dr, prompt.tolist(), g


def _advance(dr, toks, seqs, n, g, vocab):
    B, K = toks.shape
    res = AcceptResult(tokens=torch.zeros(B, K + 1, dtype=torch.int32, device="cuda"),
                       num_accepted=torch.tensor(n, dtype=torch.int32, device="cuda"),
                       eos=torch.zeros(B, dtype=torch.bool, device="cuda"))
    finals = torch.randint(0, vocab, (B,), generator=g).tolist()
    for b in range(B):
        emitted = toks[b, : n[b]].tolist() + [finals[b]]
        res.tokens[b, : len(emitted)] = torch.tensor(emitted, dtype=torch.int32)
        seqs[b] = seqs[b] + emitted
    dr.advance(res, [x + 1 for x in n])


@pytest.mark.parametrize("cfg", [SMALL_INT4, TINY_DRAFT], ids=["int4_gqa", "tiny_fp16"])
def test_draft_rounds_match_fp32_oracle(cfg):
    B, S0, K = 3, 21, 4
    model, dr, seqs, g = _setup(cfg, B, S0, K, seed=5)
    accepts = [[0, K, 2], [K, 1, 0], [3, 0, K]]
    checked = 0
    for r in range(3):
        toks, logits = dr.draft()
        torch.cuda.synchronize()
        assert int(dr.status.item()) == 0
        toks, logits = toks.cpu(), logits.cpu()
        for b in range(B):
            S = len(seqs[b])
            full = torch.tensor([seqs[b] + toks[b].tolist()]).cuda()
            ref = llama_ref.forward_full(model, full)[0].cpu()
            clear = _check_logits(logits[b], ref[S - 1: S - 1 + K])
            # greedy: each draft is the argmax of its own row
            assert torch.equal(toks[b][clear].long(), logits[b].float().argmax(-1)[clear])
            checked += int(clear.sum())
        _advance(dr, toks, seqs, accepts[r], g, cfg.vocab)
    assert checked > 0


def test_stochastic_draft_uses_uniform_j_for_token_j():
    B, S0, K = 4, 17, 3
    model, dr, seqs, g = _setup(SMALL_INT4, B, S0, K, seed=9, greedy=False, temperature=0.8)
    u = torch.rand(B, K, generator=g).cuda()
    toks, logits = dr.draft(u)
    torch.cuda.synchronize()
    empty = torch.zeros(B, 0, dtype=torch.int32, device="cuda")
    for j in range(K):
        r = accept_sample(None, logits[:, j: j + 1].clone(), empty, u[:, j: j + 1].contiguous(), temperature=0.8)
        assert torch.equal(r.tokens[:, 0], toks[:, j])


def test_graph_rounds_match_eager():
    B, S0, K = 3, 25, 4
    outs = []
    for use_graph in (False, True):
        model, dr, seqs, g = _setup(SMALL_INT4, B, S0, K, seed=11, use_graph=use_graph)
        rounds = []
        for r in range(4):
            toks, logits = dr.draft()
            rounds.append((toks.clone().cpu(), logits.clone().float().cpu()))
            _advance(dr, toks.cpu(), seqs, [[1, K, 0], [K, 2, 3], [0, 0, K], [2, 2, 2]][r], g, SMALL_INT4.vocab)
        torch.cuda.synchronize()
        assert (dr.graph is not None) == use_graph
        outs.append(rounds)
    compared = 0
    for (t0, l0), (t1, l1) in zip(*outs):
        scale = max(1.0, l0.abs().max().item())
        assert (l0 - l1).abs().max().item() / scale <= 2e-2
        top2 = l0.topk(2, dim=-1).values
        clear = (top2[..., 0] - top2[..., 1]) > 2e-2 * scale
        assert torch.equal(t0[clear], t1[clear])
        compared += 1
        if not torch.equal(t0, t1):  # a near-tie went the other way: the histories diverge from here
            break
    assert compared >= 1
