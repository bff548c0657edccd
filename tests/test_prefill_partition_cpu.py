"""The tcgen05 prefill kernel's work split, restated on the host.

The kernel (csrc/nie_attn_prefill.cu, PfSegIter) lays segments end to end,
each costing kPfSegCost plus its key tiles, and gives CTA b the cost range
[b W, (b+1) W).  A segment cut by range boundaries is merged by the CTA where
it begins, from partials of the CTAs after it.  These checks pin the facts
the in-kernel merge relies on: every key tile is processed exactly once,
every CTA that touches a segment processes at least one tile of it, a cut
segment has exactly one merging CTA (first tile, not the last), and its
producers are exactly CTAs c0+1 .. c1 with c1 = (start + n - 1) // W, each
on its first segment.
"""

import random

SEG_COST = 3  # kPfSegCost


def _walk(n_kts, hq, grid):
    cost = [n + SEG_COST if n > 0 else 0 for n in n_kts]
    cum = [0]
    for c in cost:
        cum.append(cum[-1] + c)
    units = len(n_kts)
    total = hq * cum[units]
    if total == 0:
        return {}, 0
    W = -(-total // grid)
    touched = {}
    for b in range(grid):
        lo, hi = b * W, min(total, (b + 1) * W)
        if lo >= hi:
            continue
        left, right = 0, units - 1  # largest unit with hq * cum[u] <= lo
        while left < right:
            mid = (left + right + 1) >> 1
            if hq * cum[mid] <= lo:
                left = mid
            else:
                right = mid - 1
        u = left
        d = cum[u + 1] - cum[u]
        n = d - SEG_COST if d > 0 else 0
        h = (lo - hq * cum[u]) // d if d > 0 else 0
        start = hq * cum[u] + h * d + SEG_COST
        k = 0
        while lo < hi and start < hi:
            tlo, thi = max(lo, start) - start, min(hi, start + n) - start
            touched.setdefault((u, h), []).append({"cta": b, "tlo": tlo, "thi": thi, "n": n, "k": k, "start": start})
            h += 1
            if h < hq:
                start += d
            else:
                h = 0
                u += 1
                while u < units and cum[u + 1] == cum[u]:
                    u += 1
                if u >= units:
                    break
                d = cum[u + 1] - cum[u]
                n = d - SEG_COST
                start = hq * cum[u] + SEG_COST
            k += 1
    return touched, W


def test_cut_segments_have_one_merger_and_the_next_ctas_as_producers():
    rng = random.Random(1)
    for _ in range(600):
        units = rng.randint(1, 40)
        n_kts = [rng.choice([0, rng.randint(1, 200)]) for _ in range(units)]
        hq = rng.choice([1, 4, 32])
        grid = rng.choice([1, 7, 148, 296])
        touched, W = _walk(n_kts, hq, grid)
        assert len(touched) == hq * sum(1 for n in n_kts if n > 0)
        for parts in touched.values():
            n = parts[0]["n"]
            assert sum(p["thi"] - p["tlo"] for p in parts) == n  # each tile once
            assert all(p["thi"] > p["tlo"] for p in parts)
            if len(parts) == 1:
                assert parts[0]["tlo"] == 0 and parts[0]["thi"] == n  # whole: written directly
                continue
            mergers = [p for p in parts if p["tlo"] == 0 and p["thi"] < n]
            producers = [p for p in parts if p["tlo"] > 0]
            assert len(mergers) == 1 and len(producers) == len(parts) - 1
            c0 = mergers[0]["cta"]
            c1 = (mergers[0]["start"] + n - 1) // W
            assert sorted(p["cta"] for p in producers) == list(range(c0 + 1, c1 + 1))
            assert all(p["k"] == 0 for p in producers)
