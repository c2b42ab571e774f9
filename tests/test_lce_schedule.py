"""The closed-form list schedule of the linear + CE grouped GEMM launch (csrc/linear_ce.cu,
`sched_tile`), restated here and checked on CPU.

The grouped dW / dH launch mixes short-K and long-K tiles.  Pairs take the long tiles round robin,
then each pair takes the next short tile when it becomes free.  With two tile costs the order in
which pairs become free has a closed form, so every role of a CTA pair computes its own tile
sequence with no exchange.  These tests check that the arithmetic the kernel uses equals a
heap-based list scheduler (ties broken by the lower pair) and hands out every tile exactly once.
The GPU tests check the kernel's results, which would be wrong if a tile were skipped or doubled.
"""
import heapq
import itertools

import pytest


def sched_tile(n_long, n_short, c_long, c_short, pair, npairs, k):
    """The kernel's formula: ('L', i) or ('S', i) for this pair's k-th turn, or None."""
    q, r = divmod(n_long, npairs)
    nl = q + (1 if pair < r else 0)
    if k < nl:
        return ("L", pair + k * npairs)
    tau = nl * c_long + (k - nl) * c_short
    xa, xb = tau - (q + 1) * c_long, tau - q * c_long
    na = 0 if xa <= 0 else (xa + c_short - 1) // c_short
    nb = 0 if xb <= 0 else (xb + c_short - 1) // c_short
    s = r * na + (npairs - r) * nb
    if xa >= 0 and xa % c_short == 0:
        s += min(pair, r)
    if xb >= 0 and xb % c_short == 0:
        s += max(0, pair - r)
    return ("S", s) if s < n_short else None


def list_schedule(n_long, n_short, c_long, c_short, npairs):
    free = [(0, p) for p in range(npairs)]
    out = {p: [] for p in range(npairs)}
    for kind, i, c in [("L", i, c_long) for i in range(n_long)] + [("S", i, c_short) for i in range(n_short)]:
        t, p = heapq.heappop(free)
        out[p].append((kind, i))
        heapq.heappush(free, (t + c, p))
    return out


def per_pair(n_long, n_short, c_long, c_short, npairs):
    got = {}
    for p in range(npairs):
        seq, k = [], 0
        while (t := sched_tile(n_long, n_short, c_long, c_short, p, npairs, k)) is not None:
            seq.append(t)
            k += 1
            assert k <= n_long + n_short
        got[p] = seq
    return got


CASES = list(itertools.product([0, 1, 5, 48, 74, 192, 200], [0, 3, 100, 591], [790, 260, 100], [260, 68, 100],
                               [74, 7, 1]))


@pytest.mark.parametrize("n_long,n_short,c_long,c_short,npairs",
                         [c for c in CASES if c[2] >= c[3]])
def test_closed_form_equals_list_scheduling(n_long, n_short, c_long, c_short, npairs):
    got = per_pair(n_long, n_short, c_long, c_short, npairs)
    assert got == list_schedule(n_long, n_short, c_long, c_short, npairs)
    longs = sorted(i for seq in got.values() for kind, i in seq if kind == "L")
    shorts = sorted(i for seq in got.values() for kind, i in seq if kind == "S")
    assert longs == list(range(n_long)) and shorts == list(range(n_short))


def test_benchmarked_chunk_is_balanced():
    """16384-row chunk, V = 50304, D = 768: 192 dH tiles of 786 K blocks and 591 dW tiles of 256
    (+4 per tile) over 74 pairs; the busiest pair carries at most 2 % over the mean."""
    c_long, c_short = 786 + 4, 256 + 4
    got = per_pair(192, 591, c_long, c_short, 74)
    loads = [sum(c_long if kind == "L" else c_short for kind, _ in seq) for seq in got.values()]
    assert max(loads) <= 1.02 * sum(loads) / len(loads)
