"""Seeded synthetic inputs for the benchmark workloads.

No dataset ships with the reference and none is reachable here, so every
workload is generated from a fixed seed with numpy's PCG64 (same bits on every
machine with the same numpy).  Shapes and value distributions follow the
benchmark configurations:

* ``wkv_op_inputs``: the isolated WKV-7 scan op.  r, k, v, w_raw ~ N(0, 1);
  a = sigmoid(N(0, 1)); kk = L2-normalised N(0, 1) per head; the op inputs are
  ``a_op = -kk`` and ``b_op = kk * a``, the mapping ``RWKV7TimeMix._inputs_impl``
  uses (``yufmusicgen/model.py:121-122``).
* ``rosa_op_inputs``: the ROSA scan op.  cand, write, read_gate ~ N(0, 1);
  decay = sigmoid(N(0, 1)); direction = normalised N(0, 1).
* ``tiny_ids``: batch x T ids, first 32 uniform in [0, 256) (a UTF-8 byte
  caption prefix), the rest uniform in [256, 512).
* ``zipf_ids``: an optional 64-token byte prefix, then ids over
  [256, vocab) with rank-k probability proportional to k^-1.1 and a seeded
  shuffled rank -> id map.
"""

from __future__ import annotations

import numpy as np


def wkv_op_inputs(B: int, T: int, H: int, N: int, seed: int = 0, with_state: bool = False):
    rng = np.random.default_rng(seed)
    shape = (B, T, H, N)
    r = rng.standard_normal(shape, dtype=np.float32)
    w = rng.standard_normal(shape, dtype=np.float32)
    k = rng.standard_normal(shape, dtype=np.float32)
    v = rng.standard_normal(shape, dtype=np.float32)
    gate = 1.0 / (1.0 + np.exp(-rng.standard_normal(shape, dtype=np.float32)))
    kk = rng.standard_normal(shape, dtype=np.float32)
    kk /= np.maximum(np.linalg.norm(kk, axis=-1, keepdims=True), 1e-12)
    a = (-kk).astype(np.float32)
    b = (kk * gate).astype(np.float32)
    s0 = None
    if with_state:
        s0 = (0.5 * rng.standard_normal((B, H, N, N))).astype(np.float32)
    return dict(r=r, w=w, k=k, v=v, a=a, b=b, s0=s0)


def rosa_op_inputs(B: int, T: int, R: int, seed: int = 0, with_state: bool = False):
    rng = np.random.default_rng(seed)
    cand = rng.standard_normal((B, T, R), dtype=np.float32)
    write = rng.standard_normal((B, T, R), dtype=np.float32)
    read_gate = rng.standard_normal((B, T, R), dtype=np.float32)
    decay = (1.0 / (1.0 + np.exp(-rng.standard_normal(R)))).astype(np.float32)
    direction = rng.standard_normal(R).astype(np.float32)
    direction /= max(float(np.linalg.norm(direction)), 1e-12)
    m0 = rng.standard_normal((B, R), dtype=np.float32) if with_state else np.zeros((B, R), np.float32)
    return dict(cand=cand, write=write, read_gate=read_gate, decay=decay, direction=direction, m0=m0)


def tiny_ids(B: int = 2, T: int = 256, seed: int = 0, vocab: int = 512) -> np.ndarray:
    rng = np.random.default_rng(seed)
    ids = np.empty((B, T), np.int64)
    pre = min(32, T)
    ids[:, :pre] = rng.integers(0, 256, (B, pre))
    if T > pre:
        ids[:, pre:] = rng.integers(256, vocab, (B, T - pre))
    return ids


def zipf_ids(B: int, T: int, seed: int, vocab: int = 20000, byte_prefix: int = 64, s: float = 1.1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    lo = 256
    n = vocab - lo
    ranks = np.arange(1, n + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    rank_to_id = rng.permutation(n) + lo
    ids = np.empty((B, T), np.int64)
    pre = min(byte_prefix, T)
    if pre:
        ids[:, :pre] = rng.integers(0, 256, (B, pre))
    if T > pre:
        draws = rng.choice(n, size=(B, T - pre), p=p)
        ids[:, pre:] = rank_to_id[draws]
    return ids
