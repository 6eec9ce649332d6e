"""Generate the committed acceptance golden vectors (run in a container that
has the reference sources; the outputs are committed, this script is the
record of how they were made).

Inputs follow BASELINE config 1 (acceptance alone on CPU): B=4, K=4,
V=32000; draft logits fp32 N(0,1)*2 (torch seed 0), shape [B,K+1,V] (the
extra row only feeds the target's bonus row); target = draft + N(0,0.5)
(seed 1); T=1.0; draft tokens drawn from softmax(draft[:, :K]) (seed 2);
uniforms U(0,1) [B,K+1] (seed 3).

Two sets of outputs are recorded:
  * "reference": the UNMODIFIED reference SpeculativeEngine::verify_candidates
    (compiled by oracle/Makefile) with rng_seed = 42 + b, the uniforms it
    drew (replayed mt19937), and its results;
  * "uniforms_seed3": the oracle restatement driven by the seed-3 uniforms.
Probabilities come from the oracle's fixed-order fp32 softmax.
"""
import hashlib
import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))
import oracle  # noqa: E402

B, K, V, T = 4, 4, 32000, 1.0


def cfg1_inputs():
    g0 = torch.Generator().manual_seed(0)
    draft = torch.randn(B, K + 1, V, generator=g0) * 2.0
    g1 = torch.Generator().manual_seed(1)
    target = draft + torch.randn(B, K + 1, V, generator=g1) * 0.5
    g2 = torch.Generator().manual_seed(2)
    probs = torch.softmax(draft[:, :K] / T, dim=-1)
    tokens = torch.multinomial(probs.reshape(B * K, V), 1, generator=g2).reshape(B, K).to(torch.int32)
    g3 = torch.Generator().manual_seed(3)
    u = torch.rand(B, K + 1, generator=g3)
    return draft.numpy(), target.numpy(), tokens.numpy(), u.numpy()


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    draft, target, tokens, u = cfg1_inputs()
    dp = oracle.softmax_rows(draft[:, :K], T)
    tp = oracle.softmax_rows(target, T)
    eos = 2  # a real id that is unlikely to be drawn; EOS paths have their own tests
    ref = []
    for b in range(B):
        seed = 42 + b
        tok, na, ef = oracle.ref_verify(seed, tokens[b], dp[b], tp[b], eos)
        if na > 0 and tok[na - 1] == eos:
            used = na  # accepted EOS: no further draw
        elif na == K:
            used = K + 1  # K tests + the bonus draw
        else:
            used = na + 2  # na accepted tests, the rejected test, the resample draw
        ref.append({"rng_seed": seed, "uniforms": oracle.ref_uniforms(seed, K + 1)[:used].tolist(),
                    "num_accepted": na, "tokens": tok[: na + 1].tolist(), "eos": ef})
    t3, n3, e3 = oracle.accept(tokens, dp, tp, u, eos)
    out = {
        "config": {"B": B, "K": K, "V": V, "T": T, "eos": eos},
        "inputs_sha256": digest(draft, target, tokens, u),
        "draft_tokens": tokens.tolist(),
        "uniforms_seed3": u.tolist(),
        "reference": ref,
        "uniforms_seed3_result": {"num_accepted": n3.tolist(),
                                  "tokens": [t3[b, : n3[b] + 1].tolist() for b in range(B)],
                                  "eos": e3.tolist()},
    }
    with open(os.path.join(os.path.dirname(__file__), "cfg1_accept.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out["uniforms_seed3_result"]), [r["num_accepted"] for r in ref])


if __name__ == "__main__":
    main()
