"""Pin the Philox4x32-10 restatement (oracle/philox.py) to the published
known-answer vectors of the Random123 distribution (Salmon et al., SC'11)."""

from oracle.philox import philox4x32_10, uniform

KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers():
    for ctr, key, want in KAT:
        assert philox4x32_10(ctr, key) == want


def test_uniform_range_and_mapping():
    u = uniform(0, 0, 0)
    assert u == (0x6627E8D5 >> 8) / 16777216.0
    assert all(0.0 <= uniform(7, s, q) < 1.0 for s in range(20) for q in range(5))
