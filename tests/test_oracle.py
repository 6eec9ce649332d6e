"""CPU: the acceptance oracle (oracle/accept_ref.c) against the reference.

Pins the restatement two ways: (1) against the UNMODIFIED reference
verify_candidates compiled from its sources (oracle/_ref), replaying the
reference's own mt19937 uniforms; (2) against the committed golden vectors
and the reference's own known-answer tests (tests/unit/test_speculative.py)."""
import json
import os

import numpy as np
import pytest

import oracle
from tests.helpers import cfg1_inputs, digest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "cfg1_accept.json")


def _case(rng, K, V, sharp):
    dl = rng.normal(size=(K + 1, V)).astype(np.float32) * 2
    tl = dl + rng.normal(size=(K + 1, V)).astype(np.float32) * sharp
    dp = oracle.softmax_rows(dl[:K], 1.0)
    tp = oracle.softmax_rows(tl, 1.0)
    dt = np.array([rng.choice(V, p=dp[i] / dp[i].sum()) for i in range(K)], np.int32)
    return dt, dp, tp


@pytest.mark.skipif(not oracle.ref_available(), reason="reference build absent")
def test_restatement_matches_compiled_reference():
    rng = np.random.default_rng(123)
    for t in range(200):
        K = int(rng.integers(0, 7))
        V = int(rng.integers(2, 400))
        dt, dp, tp = _case(rng, K, V, [0.0, 0.3, 1.0, 3.0][t % 4])
        eos = int(dt[0]) if (t % 5 == 0 and K > 0) else int(rng.integers(-1, V))
        seed = int(rng.integers(0, 2**32))
        tok, na, ef = oracle.ref_verify(seed, dt, dp, tp, eos)
        u = oracle.ref_uniforms(seed, K + 1)
        t2, n2, e2 = oracle.accept(dt[None], dp[None], tp[None], u[None], eos)
        assert na == n2[0] and ef == e2[0]
        assert (tok[: na + 1] == t2[0, : na + 1]).all()


@pytest.mark.skipif(not oracle.ref_available(), reason="reference build absent")
def test_greedy_restatement_matches_compiled_reference():
    rng = np.random.default_rng(7)
    for t in range(100):
        K = int(rng.integers(0, 6))
        V = int(rng.integers(2, 50))
        tp = rng.random((K + 1, V)).astype(np.float32)
        tp[:, rng.integers(0, V)] = 2.0  # forced ties with lower index
        dt = np.array([np.argmax(tp[i]) if rng.random() < 0.7 else rng.integers(0, V) for i in range(K)], np.int32)
        eos = int(rng.integers(-1, V))
        tok, na, ef = oracle.ref_verify_greedy(dt, tp, eos)
        t2, n2, e2 = oracle.accept_greedy(dt[None], tp[None], eos)
        assert na == n2[0] and ef == e2[0] and (tok[: na + 1] == t2[0, : na + 1]).all()


def test_reference_known_answer_greedy():
    # reference tests/unit/test_speculative.py:6-37
    tp = np.array([[0, 1, 0, 0, 0], [0, 0, 1, 0, 0], [0, 0, 0, 0, 1], [1, 0, 0, 0, 0]], np.float32)
    tok, na, ef = oracle.accept_greedy(np.array([[1, 2, 3]]), tp[None], 0)
    assert na[0] == 2 and tok[0, :2].tolist() == [1, 2] and tok[0, 2] == 4
    # :40-57, full acceptance with bonus = EOS
    tp = np.array([[0, 1, 0], [0, 0, 1], [1, 0, 0]], np.float32)
    tok, na, ef = oracle.accept_greedy(np.array([[1, 2]]), tp[None], 0)
    assert na[0] == 2 and tok[0, :2].tolist() == [1, 2] and tok[0, 2] == 0 and ef[0] == 1


def test_reference_probe_eos():
    # the probe recorded with the reference build: verify_candidates([1,2], [[.2]*5]*2,
    # [[0,1,0,0,0],[0,0,1,0,0],[1,0,0,0,0]], 0) -> 2 accepted, [1,2], final 0, eos
    dp = np.full((2, 5), 0.2, np.float32)
    tp = np.array([[0, 1, 0, 0, 0], [0, 0, 1, 0, 0], [1, 0, 0, 0, 0]], np.float32)
    u = np.array([0.5, 0.5, 0.5], np.float32)
    tok, na, ef = oracle.accept(np.array([[1, 2]]), dp[None], tp[None], u[None], 0)
    assert na[0] == 2 and tok[0].tolist() == [1, 2, 0] and ef[0] == 1


def test_cfg1_golden_vectors():
    g = json.load(open(GOLD))
    c = g["config"]
    draft, target, tokens, u = cfg1_inputs(c["B"], c["K"], c["V"], c["T"])
    assert digest(draft.numpy(), target.numpy(), tokens.numpy(), u.numpy()) == g["inputs_sha256"]
    K = c["K"]
    dp = oracle.softmax_rows(draft[:, :K].numpy(), c["T"])
    tp = oracle.softmax_rows(target.numpy(), c["T"])
    # (a) the reference run with its own RNG, replayed through the explicit-uniform contract
    for b, r in enumerate(g["reference"]):
        uu = np.zeros(K + 1, np.float32)
        uu[: len(r["uniforms"])] = r["uniforms"]
        tok, na, ef = oracle.accept(tokens[b : b + 1].numpy(), dp[b : b + 1], tp[b : b + 1], uu[None], c["eos"])
        assert na[0] == r["num_accepted"] and tok[0, : na[0] + 1].tolist() == r["tokens"] and ef[0] == r["eos"]
    # (b) the seed-3 uniforms
    tok, na, ef = oracle.accept(tokens.numpy(), dp, tp, u.numpy(), c["eos"])
    res = g["uniforms_seed3_result"]
    assert na.tolist() == res["num_accepted"]
    assert [tok[b, : na[b] + 1].tolist() for b in range(c["B"])] == res["tokens"]


def test_tree_restatement_branching_one_equals_chain():
    """The tree walk (no reference counterpart) must reduce exactly to the
    pinned chain restatement when every node has a single child."""
    rng = np.random.default_rng(7)
    for t in range(200):
        K = int(rng.integers(0, 7))
        V = int(rng.integers(2, 300))
        dt, dp, tp = _case(rng, K, V, [0.0, 0.3, 1.0, 3.0][t % 4])
        eos = int(dt[0]) if (t % 5 == 0 and K > 0) else -1
        u = rng.random(K + 1).astype(np.float32)
        tok, na, ef = oracle.accept(dt[None], dp[None], tp[None], u[None], eos)
        par = np.maximum(np.arange(-1, K), 0).astype(np.int32)
        ttok = np.concatenate([[0], dt]).astype(np.int32)
        dp_tree = np.concatenate([dp, np.full((1, V), 1.0 / V, np.float32)]) if K else np.full((1, V), 1.0 / V, np.float32)
        path, toks, n2, e2 = oracle.accept_tree(par, ttok, dp_tree, tp, u, eos)
        assert n2 == na[0] and e2 == ef[0]
        assert toks == tok[0, : na[0] + 1].tolist()
        assert path == list(range(n2 + 1))
        gtok, gna, gef = oracle.accept_greedy(dt[None], tp[None], eos)
        path, toks, n2, e2 = oracle.accept_tree(par, ttok, None, tp, None, eos, greedy=True)
        assert n2 == gna[0] and e2 == gef[0] and toks == gtok[0, : n2 + 1].tolist()
