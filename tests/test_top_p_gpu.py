"""GPU: the optional nucleus (top-p) filter on the bonus draw.

The reference Python engine filters the bonus token's distribution with
top-p (cudaforge/speculative.py:58-84, :188-195); its C++ verifier has no
top-p, which is the parity-pinned default here (top_p=None).  With
top_p in (0, 1) the kernel keeps every token whose probability mass strictly
above it is <= top_p, renormalises, and draws with the same exact inverse
CDF.  Not parity-pinned (the reference draw uses torch.multinomial); tested
here against a float64 restatement of that rule: the kept set, the drawn
token (away from float32 rounding boundaries), the empirical distribution,
and that top_p=None / 1.0 leave the pinned path untouched."""
import numpy as np
import pytest
import torch

import oracle
from cudaforge_b200.accept import accept_sample

pytestmark = pytest.mark.gpu


def _nucleus(logits64, T, top_p):
    p = np.exp((logits64 - logits64.max()) / T)
    p /= p.sum()
    order = np.argsort(-p, kind="stable")
    excl = np.concatenate([[0.0], np.cumsum(p[order])[:-1]])
    keep = np.zeros_like(p, dtype=bool)
    keep[order[excl <= top_p]] = True
    q = np.where(keep, p, 0.0)
    return keep, q / q.sum(), excl


@pytest.mark.parametrize("top_p", [0.3, 0.75, 0.95])
def test_bonus_draw_follows_the_nucleus_rule(top_p):
    B, V, T = 512, 3000, 0.9
    g = torch.Generator().manual_seed(int(top_p * 100))
    logits = torch.randn(B, 1, V, generator=g) * 2.5
    u = torch.rand(B, 1, generator=g)
    res = accept_sample(None, logits.cuda(), torch.zeros(B, 0, dtype=torch.int32).cuda(), u.cuda(), temperature=T,
                        top_p=top_p)
    torch.cuda.synchronize()
    tok = res.tokens[:, 0].cpu().numpy()
    checked = 0
    for b in range(B):
        keep, q, excl = _nucleus(logits[b, 0].double().numpy(), T, top_p)
        assert keep[tok[b]], b
        # the token that crosses top_p (last kept in descending order) and the first dropped one
        ex = np.sort(excl)
        k = int(np.searchsorted(ex, top_p, side="right"))
        if abs(ex[k - 1] - top_p) < 1e-5 or (k < len(ex) and abs(ex[k] - top_p) < 1e-5):
            continue  # the kept set is within float32 rounding of top_p
        cum = np.cumsum(q)
        r = float(u[b, 0])
        want = int(np.searchsorted(cum, r, side="left"))
        lo_edge = cum[want - 1] if want > 0 else 0.0
        if want < V and (cum[want] - r < 1e-5 or r - lo_edge < 1e-5):
            continue  # the uniform sits within float32 rounding of a CDF step
        assert tok[b] == want, b
        checked += 1
    assert checked > B // 2


def test_nucleus_distribution():
    B, V, T, top_p = 40000, 40, 1.0, 0.8
    g = torch.Generator().manual_seed(5)
    row = torch.randn(V, generator=g) * 1.5
    logits = row.view(1, 1, V).expand(B, 1, V).contiguous()
    u = torch.rand(B, 1, generator=g)
    res = accept_sample(None, logits.cuda(), torch.zeros(B, 0, dtype=torch.int32).cuda(), u.cuda(), temperature=T,
                        top_p=top_p)
    torch.cuda.synchronize()
    counts = np.bincount(res.tokens[:, 0].cpu().numpy(), minlength=V)
    keep, q, _ = _nucleus(row.double().numpy(), T, top_p)
    assert counts[~keep].sum() == 0
    sigma = np.sqrt(B * q * (1 - q)) + 1.0
    assert (np.abs(counts - B * q) < 6 * sigma).all()


def test_bonus_after_full_acceptance_and_off_switch():
    """d == t: every draft is accepted, so the draw is the bonus from row K and
    top-p applies; top_p None and 1.0 give the pinned C++ semantics."""
    B, K, V = 64, 3, 5000
    g = torch.Generator().manual_seed(9)
    d = torch.randn(B, K + 1, V, generator=g) * 2.0
    dt = torch.multinomial(torch.softmax(d[:, :K].reshape(-1, V), -1), 1, generator=g).reshape(B, K)
    u = torch.rand(B, K + 1, generator=g)
    res = accept_sample(d[:, :K].cuda(), d.cuda(), dt.cuda(), u.cuda(), top_p=0.5)
    torch.cuda.synchronize()
    assert (res.num_accepted.cpu() == K).all()
    for b in range(B):
        keep, _, _ = _nucleus(d[b, K].double().numpy(), 1.0, 0.5)
        assert keep[int(res.tokens[b, K])]
    for off in (None, 1.0):
        r = accept_sample(d[:, :K].cuda(), d.cuda(), dt.cuda(), u.cuda(), top_p=off, export_probs=True)
        torch.cuda.synchronize()
        tok, na, _ = oracle.accept(dt.numpy().astype(np.int32), r.probs_draft.cpu().numpy(),
                                   r.probs_target.cpu().numpy(), u.numpy(), -1)
        assert (r.num_accepted.cpu().numpy() == na).all()
        for b in range(B):
            assert r.emitted(b) == tok[b, : na[b] + 1].tolist()
