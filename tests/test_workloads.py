"""The bench's roofline numerators on CPU: seeded batch totals, the useful-pair count against a
brute-force mask of the reference's band rule (runtime/attention.py:157-170), and the per-launch
FLOP / byte figures of the benchmark configurations."""

from __future__ import annotations

import numpy as np
import pytest

from packed_encoders_b200 import workloads as wl
from packed_encoders_b200.shard import band_pairs


def _mask_pairs(length: int, window: tuple[int, int], causal: bool) -> int:
    i = np.arange(length)[:, None]
    j = np.arange(length)[None, :]
    left, right = window
    ok = np.ones((length, length), dtype=bool)
    if left >= 0:
        ok &= j >= i - left
    if right >= 0:
        ok &= j <= i + right
    if causal:
        ok &= j <= i
    return int(ok.sum())


@pytest.mark.parametrize("length", [0, 1, 7, 64, 65, 130, 257])
@pytest.mark.parametrize("window,causal", [((-1, -1), False), ((64, 64), False), ((0, 0), False), ((8, -1), False),
                                           ((-1, 3), False), ((-1, -1), True), ((16, -1), True), ((5, 9), False)])
def test_band_pairs_match_mask(length, window, causal):
    assert band_pairs(length, window, causal) == _mask_pairs(length, window, causal)


def test_seeded_totals():
    assert wl.config1().tokens == 9_371
    assert wl.config2().tokens == 147_509
    assert wl.config3().tokens == 450_079
    assert wl.config5().tokens == 543_071
    assert len(wl.config3("mix").layers) == 28
    assert sum(1 for w, _ in wl.config3("mix").layers if w == (-1, -1)) == 10


@pytest.mark.parametrize("make,window,causal,flop,nbytes", [
    (wl.config2, (-1, -1), False, 19.7e9, 906e6),
    (lambda: wl.config3("global"), (-1, -1), False, 3.43e12, 3.69e9),
    (lambda: wl.config3("local"), (64, 64), False, 0.229e12, 3.69e9),
    (wl.config5, (-1, -1), True, 6.14e12, 5.56e9),
])
def test_roofline_numerators(make, window, causal, flop, nbytes):
    w = make()
    got_flop = wl.useful_flops(w.lengths, w.heads, w.head_dim, window, causal)
    got_bytes = wl.algorithmic_bytes(w.tokens, w.tokens, w.heads, w.kv_heads, w.head_dim)
    assert got_flop == pytest.approx(flop, rel=5e-3)
    assert got_bytes == pytest.approx(nbytes, rel=5e-3)
    # FLOP = 4 * pairs * H * D, pairs never above the dense L^2 per sequence.
    assert got_flop <= 4 * sum(n * n for n in w.lengths) * w.heads * w.head_dim
