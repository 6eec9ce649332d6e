"""CPU: the reference's native module surface (`cudaforge._C`) as this package
provides it (cudaforge_b200._C).

  * SpeculativeEngine: the reference's own unit tests
    (tests/unit/test_speculative.py:6-57) run through it, and random
    stochastic / greedy calls -- several calls on ONE engine, so the random
    stream carries over -- give exactly what the UNMODIFIED reference engine
    (oracle/_ref/libspec_ref.so) gives for the same seed and inputs;
  * ContinuousBatcher + ModelRunner + TokenStreamBuffer: random operation
    scripts give the same streamed outputs and queue counts as the
    UNMODIFIED reference classes (oracle/_ref/libsched_ref.so);
  * the reference's cudaforge/engine.py, loaded unchanged with
    `cudaforge._C` bound to this package, runs LLMEngine end to end (needs
    the reference checkout; skipped without it)."""
import importlib.util
import os
import sys
import types

import numpy as np
import pytest

import oracle
from cudaforge_b200 import _C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference acceptance build absent")


def test_reference_unit_tests_greedy():
    cfg = _C.SpeculativeConfig()
    cfg.gamma = 3
    eng = _C.SpeculativeEngine(cfg)
    tp = [[0.0, 1.0, 0.0, 0.0, 0.0], [0.0, 0.0, 1.0, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 0.0, 0.0]]
    r = eng.verify_candidates_greedy([1, 2, 3], tp, eos_token_id=0)
    assert r.num_accepted == 2 and r.accepted_tokens == [1, 2] and r.final_token == 4
    cfg.gamma = 2
    eng = _C.SpeculativeEngine(cfg)
    r = eng.verify_candidates_greedy([1, 2], [[0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [1.0, 0.0, 0.0]], eos_token_id=0)
    assert r.num_accepted == 2 and r.accepted_tokens == [1, 2] and r.final_token == 0 and r.end_of_sequence


def test_certain_acceptance_then_eos_final_token():
    """p(draft) = 1 under the target: both drafts accepted; the final draw is the
    certain token 0, which is the eos id."""
    eng = _C.SpeculativeEngine(_C.SpeculativeConfig())
    r = eng.verify_candidates([1, 2], [[0.2] * 5] * 2, [[0, 1, 0, 0, 0], [0, 0, 1, 0, 0], [1, 0, 0, 0, 0]], 0)
    assert (r.num_accepted, r.accepted_tokens, r.final_token, r.end_of_sequence) == (2, [1, 2], 0, True)


def test_config_roundtrip_and_errors():
    cfg = _C.SpeculativeConfig()
    assert (cfg.gamma, cfg.temperature, cfg.top_p, cfg.rng_seed) == (5, 1.0, 1.0, 42)
    cfg.gamma, cfg.temperature, cfg.top_p, cfg.rng_seed = 4, 0.5, 0.9, 7
    eng = _C.SpeculativeEngine(cfg)
    got = eng.get_config()
    assert (got.gamma, got.temperature, got.top_p, got.rng_seed) == (4, 0.5, pytest.approx(0.9), 7)
    with pytest.raises(ValueError):  # K draft rows required (speculative.cpp:59-62)
        eng.verify_candidates([1, 2], [[0.5, 0.5]], [[0.5, 0.5]] * 3, -1)
    with pytest.raises(ValueError):
        eng.verify_candidates([1], [[0.5, 0.5]], [[0.5, 0.5]], -1)


def _case(rng, K, V, mode):
    d = rng.normal(size=(K + 1, V)) * 2.0
    t = d + 0.3 * rng.normal(size=(K + 1, V)) if mode == "close" else (
        d.copy() if mode == "same" else rng.normal(size=(K + 1, V)) * 3.0)
    dp = np.exp(d - d.max(-1, keepdims=True)).astype(np.float32)
    dp /= dp.sum(-1, keepdims=True)
    tp = np.exp(t - t.max(-1, keepdims=True)).astype(np.float32)
    tp /= tp.sum(-1, keepdims=True)
    toks = np.array([rng.choice(V, p=dp[i].astype(np.float64) / dp[i].astype(np.float64).sum()) for i in range(K)],
                    dtype=np.int32)
    return toks, dp[:K], tp


@needs_ref
@pytest.mark.parametrize("seed", [0, 1, 42, 2**40 + 3])
@pytest.mark.parametrize("mode", ["close", "far", "same"])
def test_stream_matches_reference_engine(seed, mode):
    rng = np.random.default_rng(seed % 1000 + len(mode))
    B, K, V = 8, 4, 700
    cases = [_case(rng, K, V, mode) for _ in range(B)]
    dt = np.stack([c[0] for c in cases])
    dp = np.stack([c[1] for c in cases])
    tp = np.stack([c[2] for c in cases])
    eos = int(dt[2, 1])
    ref_tok, ref_na, ref_eos = oracle.ref_verify_stream(seed, dt, dp, tp, eos)
    cfg = _C.SpeculativeConfig()
    cfg.rng_seed = seed
    eng = _C.SpeculativeEngine(cfg)
    for b in range(B):
        r = eng.verify_candidates(dt[b].tolist(), dp[b].tolist(), tp[b].tolist(), eos)
        assert r.num_accepted == ref_na[b], b
        assert r.accepted_tokens + [r.final_token] == ref_tok[b, : ref_na[b] + 1].tolist(), b
        assert r.end_of_sequence == bool(ref_eos[b]), b


@needs_ref
def test_set_config_keeps_the_stream():
    """set_config replaces the configuration only; the engine's stream is not
    reseeded (speculative.h:70-73), so later calls match the reference stream."""
    rng = np.random.default_rng(5)
    B, K, V = 4, 3, 200
    cases = [_case(rng, K, V, "far") for _ in range(B)]
    dt, dp, tp = (np.stack([c[i] for c in cases]) for i in range(3))
    ref_tok, ref_na, _ = oracle.ref_verify_stream(9, dt, dp, tp, -1)
    cfg = _C.SpeculativeConfig()
    cfg.rng_seed = 9
    eng = _C.SpeculativeEngine(cfg)
    out = []
    for b in range(B):
        other = _C.SpeculativeConfig()
        other.rng_seed = 1234 + b
        eng.set_config(other)
        r = eng.verify_candidates(dt[b].tolist(), dp[b].tolist(), tp[b].tolist(), -1)
        out.append(r.accepted_tokens + [r.final_token])
    assert out == [ref_tok[b, : ref_na[b] + 1].tolist() for b in range(B)]


@needs_ref
def test_greedy_matches_reference():
    rng = np.random.default_rng(3)
    for trial in range(30):
        K, V = int(rng.integers(0, 6)), int(rng.integers(2, 300))
        tp = rng.random((K + 1, V)).astype(np.float32)
        tp[:, rng.integers(0, V)] = tp.max() if trial % 3 == 0 else tp[:, 0]  # ties
        am = tp.argmax(-1)
        dt = am[:K].astype(np.int32).copy()
        if K and trial % 2:
            dt[int(rng.integers(0, K))] = int(rng.integers(0, V))
        eos = int(am[0]) if trial % 5 == 0 else -1
        ref = oracle.ref_verify_greedy(dt, tp, eos)
        r = _C.SpeculativeEngine(_C.SpeculativeConfig()).verify_candidates_greedy(dt.tolist(), tp.tolist(), eos)
        assert r.num_accepted == ref[1]
        assert r.accepted_tokens + [r.final_token] == ref[0][: ref[1] + 1].tolist()
        assert r.end_of_sequence == bool(ref[2])


@needs_ref
def test_draw_uniforms_is_the_reference_stream():
    eng = _C.SpeculativeEngine(_C.SpeculativeConfig())
    assert np.array_equal(eng.draw_uniforms(1000), oracle.ref_uniforms(42, 1000))


# ---------------------------------------------------------------- scheduler
needs_sched = pytest.mark.skipif(not oracle.RefSched.available(), reason="reference scheduler build absent")


@needs_sched
@pytest.mark.parametrize("seed", range(8))
def test_scheduler_and_runner_match_reference(seed):
    rng = np.random.default_rng(seed)
    max_seqs, max_tok, vocab, eos = int(rng.integers(1, 6)), int(rng.integers(3, 60)), 50, 7
    ref = oracle.RefSched(max_seqs, max_tok, vocab, eos)
    batcher = _C.ContinuousBatcher(max_seqs, max_tok)
    runner = _C.ModelRunner(batcher, vocab, eos)
    next_id = 1
    for _ in range(120):
        op = rng.random()
        if op < 0.35:
            rid = next_id if rng.random() < 0.9 else max(1, next_id - 1)  # duplicates are refused
            next_id += 1
            prompt = rng.integers(0, vocab, size=int(rng.integers(0, 12))).tolist()
            mt, prio = int(rng.integers(1, 6)), int(rng.integers(0, 3))
            assert batcher.add_request(_C.Request(rid, prompt, mt, prio)) == ref.add(rid, prompt, mt, prio)
        elif op < 0.45 and next_id > 1:
            rid = int(rng.integers(1, next_id))
            runner.cancel_request(rid)
            ref.cancel(rid)
        elif op < 0.5 and next_id > 1:
            ids = rng.integers(1, next_id, size=2).tolist()
            batcher.update_requests_state(ids)
            ref.update(ids)
        else:
            assert runner.step() == ref.step()
            ours = [(o.request_id, o.token_id, o.is_final) for o in runner.get_stream_buffer().pop_all()]
            assert ours == ref.pop()
        assert (batcher.get_pending_count(), batcher.get_running_count()) == ref.counts()


def test_stream_buffer_and_request_fields():
    buf = _C.TokenStreamBuffer()
    assert buf.empty() and buf.size() == 0
    buf.push(_C.StreamOutput(3, 9, False))
    buf.push_batch([_C.StreamOutput(4, 1, True)])
    out = buf.pop_all()
    assert [(o.request_id, o.token_id, o.is_final) for o in out] == [(3, 9, False), (4, 1, True)] and buf.empty()
    r = _C.Request(5, [1, 2, 3])
    assert r.max_new_tokens == 128 and r.priority == 0 and r.state == _C.RequestState.WAITING == _C.WAITING
    r.generated_tokens.append(4)  # a copy, as pybind's vector fields are
    assert r.generated_tokens == [] and r.get_total_length() == 3 and not r.is_finished()


# ---------------------------------------------------------------- unchanged engine.py
def _reference_root():
    ref = os.environ.get("CF_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")
    return ref if os.path.isfile(os.path.join(ref, "cudaforge", "engine.py")) else None


@pytest.mark.skipif(_reference_root() is None, reason="reference checkout absent")
def test_reference_engine_py_runs_unchanged():
    path = os.path.join(_reference_root(), "cudaforge", "engine.py")
    saved = {k: sys.modules.get(k) for k in ("cudaforge", "cudaforge._C", "cudaforge.engine")}
    pkg = types.ModuleType("cudaforge")
    pkg.__path__ = []
    pkg._C = _C
    sys.modules.update({"cudaforge": pkg, "cudaforge._C": _C})
    try:
        spec = importlib.util.spec_from_file_location("cudaforge.engine", path)
        engine = importlib.util.module_from_spec(spec)
        sys.modules["cudaforge.engine"] = engine
        spec.loader.exec_module(engine)
        assert engine._HAS_NATIVE_EXTENSION
        cfg = engine.EngineConfig(num_layers=2, num_kv_heads=2, head_dim=16, vocab_size=100, eos_token_id=2,
                                  total_gpu_blocks=64, max_num_seqs=4, max_num_batched_tokens=64)
        eng = engine.LLMEngine(cfg)
        a = eng.add_request([5, 6, 7], engine.SamplingParams(max_tokens=4))
        b = eng.add_request([97, 98], engine.SamplingParams(max_tokens=10))
        c = eng.add_request([10, 11], engine.SamplingParams(max_tokens=3, stop_token_ids={13}))
        got = {a: [], b: [], c: []}
        finals = set()
        for _ in range(12):
            for out in eng.step():
                got[out.request_id].append(out.token_id)
                if out.is_final:
                    finals.add(out.request_id)
        # the reference runner's token rule: last + 1 (mod vocab), final at max_tokens, EOS or a stop token
        assert got[a] == [8, 9, 10, 11]
        assert got[b] == [99, 0, 1, 2]                  # token 2 is the EOS id
        assert got[c] == [12, 13]                       # 13 is a stop token
        assert finals == {a, b, c}
        st = eng.get_stats()
        assert st.active_sequences_count == 0 and st.free_blocks == st.total_blocks
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


@pytest.mark.gpu
def test_verify_batch_on_gpu_uses_the_engine_stream():
    """The batched entry point runs the GPU acceptance kernel with uniforms
    drawn from the engine's own stream (sequence-major); fed the kernel's
    exported probabilities and those uniforms, the oracle decides identically."""
    import torch
    B, K, V = 16, 4, 5000
    g = torch.Generator().manual_seed(2)
    d = torch.randn(B, K + 1, V, generator=g) * 2
    t = d + 0.4 * torch.randn(B, K + 1, V, generator=g)
    dt = torch.multinomial(torch.softmax(d[:, :K].reshape(-1, V), -1), 1, generator=g).reshape(B, K).to(torch.int32)
    cfg = _C.SpeculativeConfig()
    cfg.rng_seed = 77
    eng = _C.SpeculativeEngine(cfg)
    res = eng.verify_batch(d[:, :K].cuda(), t.cuda(), dt.cuda(), eos_token_id=-1, export_probs=True)
    torch.cuda.synchronize()
    u = oracle.ref_uniforms(77, B * (K + 1)).reshape(B, K + 1) if oracle.ref_available() else None
    if u is not None:
        tok, na, _ = oracle.accept(dt.numpy(), res.probs_draft.cpu().numpy(), res.probs_target.cpu().numpy(), u, -1)
        assert (res.num_accepted.cpu().numpy() == na).all()
        for b in range(B):
            assert res.emitted(b) == tok[b, : na[b] + 1].tolist()
    # the block of B*(K+1) draws was consumed: the next draw continues the stream
    nxt = eng.draw_uniforms(1)
    if oracle.ref_available():
        assert nxt[0] == oracle.ref_uniforms(77, B * (K + 1) + 1)[-1]
