"""GPU parity of the fused acceptance kernel (cf_accept_sample) against the
CPU oracle, which is itself pinned to the reference verify_candidates.

Contract: the kernel exports the fp32 probabilities it decided on; fed those
probabilities and the same uniforms, the oracle must return bit-identical
accepted counts, token ids and EOS flags.  Separately the probabilities must
match torch fp32 softmax(logits / T) within rtol 1e-5 (atol 1e-12)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from cudaforge_b200.accept import accept_sample
from tests.helpers import cfg1_inputs

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "cfg1_accept.json")


def _check_parity(res, draft_tokens, uniforms, eos, greedy=False):
    dt = draft_tokens.cpu().numpy().astype(np.int32)
    tp = res.probs_target.cpu().numpy()
    if greedy:
        tok, na, ef = oracle.accept_greedy(dt, tp, eos)
    else:
        dp = res.probs_draft.cpu().numpy()
        tok, na, ef = oracle.accept(dt, dp, tp, uniforms.cpu().numpy(), eos)
    gna = res.num_accepted.cpu().numpy()
    gtok = res.tokens.cpu().numpy()
    geos = res.eos.cpu().numpy().astype(np.uint8)
    assert (gna == na).all(), (gna, na)
    assert (geos == ef).all(), (geos, ef)
    for b in range(dt.shape[0]):
        assert gtok[b, : na[b] + 1].tolist() == tok[b, : na[b] + 1].tolist(), b
    return na


def test_cfg1_golden_and_parity():
    g = json.load(open(GOLD))
    c = g["config"]
    K = c["K"]
    draft, target, tokens, u = cfg1_inputs(c["B"], c["K"], c["V"], c["T"])
    res = accept_sample(draft[:, :K].cuda(), target.cuda(), tokens.cuda(), u.cuda(),
                        temperature=c["T"], eos_token_id=c["eos"], export_probs=True)
    torch.cuda.synchronize()
    _check_parity(res, tokens, u, c["eos"])
    # the committed golden outputs (decided on the oracle's own softmax)
    want = g["uniforms_seed3_result"]
    assert res.num_accepted.cpu().tolist() == want["num_accepted"]
    assert [res.emitted(b) for b in range(c["B"])] == want["tokens"]
    # probabilities vs torch fp32 softmax
    ref_t = torch.softmax(target / c["T"], dim=-1)
    torch.testing.assert_close(res.probs_target.cpu(), ref_t, rtol=1e-5, atol=1e-12)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,K,V", [(1, 1, 7), (3, 4, 1000), (5, 5, 32000), (2, 6, 4099), (8, 0, 513)])
@pytest.mark.parametrize("mode", ["close", "far", "same"])
def test_fuzz_parity(dtype, B, K, V, mode):
    g = torch.Generator(device="cpu").manual_seed(B * 1000 + K * 10 + V)
    d = torch.randn(B, K + 1, V, generator=g) * 2.0
    if mode == "close":
        t = d + 0.3 * torch.randn(B, K + 1, V, generator=g)
    elif mode == "far":
        t = torch.randn(B, K + 1, V, generator=g) * 3.0
    else:  # identical distributions: always accept, residual fallback paths
        t = d.clone()
    dtoks = torch.multinomial(torch.softmax(d[:, :K].reshape(-1, V), -1), 1, generator=g).reshape(B, K) if K else torch.zeros(B, 0, dtype=torch.int64)
    u = torch.rand(B, K + 1, generator=g)
    T = 0.8 if mode == "close" else 1.0
    for eos in (-1, int(dtoks[0, 0]) if K else 0):
        res = accept_sample(d[:, :K].to(dtype).cuda(), t.to(dtype).cuda(), dtoks.cuda(), u.cuda(),
                            temperature=T, eos_token_id=eos, export_probs=True)
        torch.cuda.synchronize()
        _check_parity(res, dtoks, u, eos)


def test_residual_fallback_to_target():
    # p == q exactly except at the draft token => residual sum <= 1e-6 path
    B, K, V = 2, 2, 300
    d = torch.zeros(B, K + 1, V)
    d[:, :, 5] = 4.0
    t = d.clone()
    t[:, :, 5] = 3.9  # target puts slightly less mass on token 5
    dt = torch.full((B, K), 5, dtype=torch.int32)
    u = torch.full((B, K + 1), 0.999)
    res = accept_sample(d[:, :K].cuda(), t.cuda(), dt.cuda(), u.cuda(), export_probs=True)
    torch.cuda.synchronize()
    na = _check_parity(res, dt, u, -1)
    assert (na == 0).all()


def test_strided_and_misaligned_views():
    B, K, V = 3, 3, 1001
    g = torch.Generator().manual_seed(5)
    big = torch.randn(B, 2 * K + 3, V + 3, generator=g).cuda()
    d = big[:, 1 : K + 1, 1 : V + 1]      # row stride V+3, offset by one element
    t = big[:, K + 1 : 2 * K + 2, 2 : V + 2]
    dt = torch.randint(0, V, (B, K), generator=g)
    u = torch.rand(B, K + 1, generator=g)
    res = accept_sample(d, t, dt.cuda(), u.cuda(), export_probs=True)
    torch.cuda.synchronize()
    _check_parity(res, dt, u, -1)


def test_greedy_known_answers_and_fuzz():
    # reference tests/unit/test_speculative.py:6-37 fed as log-probabilities
    tp = torch.tensor([[0, 1, 0, 0, 0], [0, 0, 1, 0, 0], [0, 0, 0, 0, 1], [1, 0, 0, 0, 0]], dtype=torch.float32)
    res = accept_sample(None, tp.log()[None].cuda(), torch.tensor([[1, 2, 3]]).cuda(), greedy=True, eos_token_id=0)
    assert res.num_accepted.item() == 2 and res.emitted(0) == [1, 2, 4]
    tp = torch.tensor([[0, 1, 0], [0, 0, 1], [1, 0, 0]], dtype=torch.float32)
    res = accept_sample(None, tp.log()[None].cuda(), torch.tensor([[1, 2]]).cuda(), greedy=True, eos_token_id=0)
    assert res.num_accepted.item() == 2 and res.emitted(0) == [1, 2, 0] and bool(res.eos.item())
    for dtype in (torch.float32, torch.bfloat16):
        g = torch.Generator().manual_seed(11)
        B, K, V = 6, 5, 32000
        t = (torch.randn(B, K + 1, V, generator=g) * 3).to(dtype)
        am = t.float().argmax(-1)
        dt = am[:, :K].clone()
        dt[1, 2] = (dt[1, 2] + 1) % V
        dt[3, 0] = (dt[3, 0] + 7) % V
        res = accept_sample(None, t.cuda(), dt.cuda(), greedy=True, export_probs=True, eos_token_id=int(am[4, 1]))
        torch.cuda.synchronize()
        _check_parity(res, dt, None, int(am[4, 1]), greedy=True)


def test_out_of_range_draft_token_flags_sequence():
    B, K, V = 2, 2, 100
    d = torch.randn(B, K + 1, V).cuda()
    dt = torch.tensor([[1, 2], [3, 100]])
    res = accept_sample(d[:, :K], d, dt.cuda(), torch.full((B, K + 1), 0.0).cuda())
    assert res.num_accepted.cpu().tolist()[1] == -1


def test_shape_errors_raise_value_error():
    d = torch.randn(2, 4, 10).cuda()
    with pytest.raises(ValueError):
        accept_sample(d[:, :2], d, torch.zeros(2, 3, dtype=torch.int32).cuda(), torch.rand(2, 4).cuda())
    with pytest.raises(ValueError):
        accept_sample(d[:, :3], d, torch.zeros(2, 3, dtype=torch.int32).cuda(), None)


@pytest.mark.parametrize("mode", ["close", "far", "same", "mixed"])
def test_cfg3_shape_parity(mode):
    """The benchmark's acceptance shape: B=64, K=5, V=128,256 bf16 logits (32
    scan chunks of 4,096 per row), stochastic and greedy."""
    B, K, V = 64, 5, 128256
    g = torch.Generator(device="cuda").manual_seed({"close": 1, "far": 2, "same": 3, "mixed": 4}[mode])
    d = torch.randn(B, K + 1, V, generator=g, device="cuda") * 2.0
    if mode == "close":
        t = d + 0.3 * torch.randn(B, K + 1, V, generator=g, device="cuda")
    elif mode == "far":
        t = torch.randn(B, K + 1, V, generator=g, device="cuda") * 3.0
    elif mode == "same":
        t = d.clone()
    else:  # per sequence a different closeness: rejections at every position
        w = torch.linspace(0.0, 2.0, B, device="cuda").view(B, 1, 1)
        t = d + w * torch.randn(B, K + 1, V, generator=g, device="cuda")
    d, t = d.to(torch.bfloat16), t.to(torch.bfloat16)
    dtoks = torch.multinomial(torch.softmax(d[:, :K].float().reshape(-1, V), -1), 1, generator=g).reshape(B, K)
    u = torch.rand(B, K + 1, generator=g, device="cuda")
    res = accept_sample(d[:, :K], t, dtoks, u, export_probs=True)
    torch.cuda.synchronize()
    na = _check_parity(res, dtoks, u, -1)
    if mode == "mixed":
        assert len(set(na.tolist())) >= 3  # several rejection positions exercised
    if mode == "far":
        res = accept_sample(None, t, dtoks, greedy=True, export_probs=True)
        torch.cuda.synchronize()
        _check_parity(res, dtoks, None, -1, greedy=True)
