"""Philox4x32-10 in plain Python -- TEST INFRASTRUCTURE ONLY.

Restates the published counter-based generator (Salmon, Moraes, Dror, Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC'11): 10 rounds of
  (c0, c1, c2, c3) -> (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0))
with M0 = 0xD2511F53, M1 = 0xCD9E8D57 and the key bumped by (0x9E3779B9, 0xBB67AE85)
after each round.  The sampler's uniform is the first output word mapped to
[0, 1) as (x >> 8) * 2^-24, with key (seed_lo, seed_hi) and counter
(step_lo, step_hi, sequence, 0).
"""

M0, M1 = 0xD2511F53, 0xCD9E8D57
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    c0, c1, c2, c3 = ctr
    k0, k1 = key
    for _ in range(10):
        p0 = M0 * c0
        p1 = M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & MASK, p1 & MASK, ((p0 >> 32) ^ c3 ^ k1) & MASK, p0 & MASK
        k0 = (k0 + W0) & MASK
        k1 = (k1 + W1) & MASK
    return c0, c1, c2, c3


def uniform(seed: int, step: int, seq: int) -> float:
    out = philox4x32_10((step & MASK, (step >> 32) & MASK, seq & MASK, 0), (seed & MASK, (seed >> 32) & MASK))
    return (out[0] >> 8) * (1.0 / 16777216.0)
