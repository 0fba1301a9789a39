"""The host pipeline's tapered head-block schedule (ltxattn.host.tapered_blocks):
pure host logic, no GPU."""
from ltxattn.host import tapered_blocks


def test_tapered_blocks_halve_down_to_the_smallest_and_cover_every_head():
    assert tapered_blocks(32) == [16, 8, 4, 2, 2]
    assert tapered_blocks(16) == [8, 4, 2, 2]
    assert tapered_blocks(4) == [2, 2]
    assert tapered_blocks(2) == [2]
    assert tapered_blocks(1) == [1]
    for h in range(1, 97):
        for smallest in (1, 2, 3):
            s = tapered_blocks(h, smallest)
            assert sum(s) == h and all(b >= 1 for b in s)
            assert all(a >= b for a, b in zip(s, s[1:]))  # never growing
