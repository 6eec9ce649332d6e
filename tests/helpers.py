"""Shared input builders for the tests (BASELINE config 1 and fuzz cases)."""
import hashlib

import numpy as np
import torch


def cfg1_inputs(B=4, K=4, V=32000, T=1.0):
    """Config 1 inputs exactly as tests/golden/make_golden.py builds them."""
    g0 = torch.Generator().manual_seed(0)
    draft = torch.randn(B, K + 1, V, generator=g0) * 2.0
    g1 = torch.Generator().manual_seed(1)
    target = draft + torch.randn(B, K + 1, V, generator=g1) * 0.5
    g2 = torch.Generator().manual_seed(2)
    probs = torch.softmax(draft[:, :K] / T, dim=-1)
    tokens = torch.multinomial(probs.reshape(B * K, V), 1, generator=g2).reshape(B, K).to(torch.int32)
    g3 = torch.Generator().manual_seed(3)
    u = torch.rand(B, K + 1, generator=g3)
    return draft, target, tokens, u


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
