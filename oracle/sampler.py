"""CPU restatement of the device sampler's rule -- TEST INFRASTRUCTURE ONLY.

The reference samples with yufmusicgen/cli/generate.py:45-56: temperature,
the top-p cut of the sorted distribution (a token is dropped when the mass
before it exceeds top_p, generate.py:52) and torch.multinomial, after masking
to MIDI ids plus EOS (generate.py:142-147).  The device sampler keeps that
rule inside the top_k most likely ids and draws by inverse CDF with a Philox
uniform u; given the same u this function picks the same id, and reports how
close the draw came to a boundary (where float rounding could decide).
"""

from __future__ import annotations

import numpy as np


def sample_rule(logits, u, temperature, top_k, top_p, mask_below=0, eos_id=2, allow_eos=True):
    """One row: returns (id, margin) -- margin is the distance of the draw
    target, and of the top-p decision, from their nearest boundary."""
    x = np.asarray(logits, np.float32) * (np.float32(1.0) / np.float32(temperature))
    allowed = np.ones(x.shape[0], bool)
    allowed[:mask_below] = False
    if allow_eos and 0 <= eos_id < x.shape[0]:
        allowed[eos_id] = True
    ids = np.flatnonzero(allowed)
    vals = x[ids].astype(np.float64)
    order = np.lexsort((ids, -vals))[:top_k]  # value descending, ties to the smaller id
    cand, v = ids[order], vals[order]
    p = np.exp(v - v[0])
    p /= p.sum()
    cum, keep, margin = 0.0, 0, np.inf
    for i in range(len(p)):
        margin = min(margin, abs(cum - top_p))
        if cum > top_p:
            break
        cum += p[i]
        keep = i + 1
    keep = max(keep, 1)
    cdf = np.cumsum(p[:keep])
    target = u * cdf[-1]
    margin = min(margin, float(np.min(np.abs(cdf - target))))
    j = int(np.searchsorted(cdf, target, side="right"))
    return int(cand[min(j, keep - 1)]), margin
