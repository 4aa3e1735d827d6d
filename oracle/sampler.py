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


# ---- the reference's own random stream (torch's CPU generator) -------------
# yufmusicgen/cli/generate.py:45-56 samples with torch.multinomial after
# torch.manual_seed (training.py:23-28).  Restated here from the published
# algorithms: MT19937 (Matsumoto & Nishimura 1998, 2002 seeding), uniforms of
# 53 bits from two words, Exp(1) keys q = -log1p(-u) rounded to float, and the
# single-sample multinomial as argmax(p / q) over the row (one key per entry,
# in the row's order).  Pinned to draws of the reference itself
# (tests/golden/sampler_torch_cpu.npz).

class MT19937:
    """MT19937 with the 2002 seeding (low 32 bits of the seed), twisted in numpy."""

    def __init__(self, seed):
        s = np.zeros(624, np.uint64)
        s[0] = seed & 0xFFFFFFFF
        for j in range(1, 624):
            p = int(s[j - 1])
            s[j] = (1812433253 * (p ^ (p >> 30)) + j) & 0xFFFFFFFF
        self.s = s.astype(np.uint32)
        self.buf = np.empty(0, np.uint32)

    def _twist(self):
        s = self.s.astype(np.uint64)
        new = np.empty(624, np.uint64)

        def part(lo, hi, nxt, far):
            y = (s[lo:hi] & 0x80000000) | (nxt & 0x7FFFFFFF)
            new[lo:hi] = far ^ (y >> 1) ^ np.where(y & 1, 0x9908B0DF, 0).astype(np.uint64)

        part(0, 227, s[1:228], s[397:624])          # j + 397 reads old words
        part(227, 454, s[228:455], new[0:227])      # j - 227 reads words twisted above
        part(454, 623, s[455:624], new[227:396])
        part(623, 624, new[0:1], new[396:397])      # s[(623 + 1) % 624] is already new
        self.s = new.astype(np.uint32)
        y = self.s.copy()
        y ^= y >> np.uint32(11)
        y ^= (y << np.uint32(7)) & np.uint32(0x9D2C5680)
        y ^= (y << np.uint32(15)) & np.uint32(0xEFC60000)
        y ^= y >> np.uint32(18)
        self.buf = np.concatenate([self.buf, y])

    def u32(self, n):
        while self.buf.size < n:
            self._twist()
        out, self.buf = self.buf[:n], self.buf[n:]
        return out

    def exponential(self, n):
        w = self.u32(2 * n).astype(np.uint64)
        c = ((w[0::2] << np.uint64(32)) | w[1::2]) & np.uint64((1 << 53) - 1)
        u = c.astype(np.float64) * (1.0 / 9007199254740992.0)
        return (-np.log1p(-u)).astype(np.float32)


_sort_lib = None


def desc_argsort(x):
    """torch.sort(descending=True)'s order of a CPU row, ties included (the
    library std::sort torch runs, built from oracle/sort_ref.cpp)."""
    global _sort_lib
    import ctypes

    from .cref import HERE, build

    if _sort_lib is None:
        path = HERE / "_build" / "liboracle_sort.so"
        if not path.exists():
            build()
        _sort_lib = ctypes.CDLL(str(path))
        _sort_lib.oracle_desc_argsort.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        _sort_lib.oracle_desc_argsort.restype = None
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape[0], np.int32)
    _sort_lib.oracle_desc_argsort(x.ctypes.data, x.shape[0], out.ctypes.data)
    return out


def _softmax32(x):
    m = np.max(x)
    e = np.exp((x - m).astype(np.float32)).astype(np.float32)
    return (e * (np.float32(1.0) / e.sum(dtype=np.float32))).astype(np.float32)


def sample_torch_cpu(logits, temperature, top_p, gen):
    """One row through sample_token's rule on the generator `gen` (MT19937)."""
    x = np.asarray(logits, np.float32)
    if temperature <= 0:
        return int(np.argmax(x))
    x = (x / np.float32(temperature)).astype(np.float32)
    order = desc_argsort(x)
    p = _softmax32(x[order])
    cum = np.cumsum(p.astype(np.float64)).astype(np.float32)
    s = np.where((cum - p) > np.float32(top_p), -np.inf, x[order]).astype(np.float32)
    p2 = _softmax32(s)
    q = gen.exponential(x.shape[0])
    return int(order[int(np.argmax(p2 / q))])
