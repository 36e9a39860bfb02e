"""The decode kernel's split of the KV stream over its persistent CTAs, restated
on the CPU (lean-infer_b200/csrc/la_decode.cu: split_from_regs, the fallback
walk, the producer's walk and the combine pass's slot lookup).

Sequence b holds units_of(ctx_b) units of 16 x (8 / Hkv) tokens; over all T
units CTA c takes [c*T/G, (c+1)*T/G). The producer and the combine pass find
a row's partial slots independently, from the lengths alone; these tests
check that they agree:
every key unit is loaded by exactly one CTA, a row held whole by one CTA is
flagged whole (written directly), and the slots the producers write for split
rows are exactly the slots the combine pass reads.
"""
import random

import pytest

TC = 16  # tokens per unit at 8 kv heads (16 x 8 / Hkv)


def units_of(ctx, tc=TC):
    return (ctx + tc - 1) // tc


def cta_start(c, T, G):
    return c * T // G


def cta_of(x, T, G):
    return ((x + 1) * G - 1) // T


def cta_schedule(lens, c, G):
    """(u0, units, b0, pb0) of CTA c, as the kernel's scheduling warp computes
    them (split_from_regs and the fallback walk)."""
    un = [units_of(x) for x in lens]
    T = sum(un)
    u0, u1 = cta_start(c, T, G), cta_start(c + 1, T, G)
    if u1 <= u0:
        return u0, 0, len(lens), T
    acc = 0
    for b, w in enumerate(un):
        if acc + w > u0:
            return u0, u1 - u0, b, acc
        acc += w
    raise AssertionError("u0 < T lies in some sequence")


def producer_walk(lens, c, G):
    """The descriptors CTA c's producer issues: (b, unit, first, last, whole, slot)."""
    u0, nu, b, pb0 = cta_schedule(lens, c, G)
    out = []
    if nu == 0:
        return out
    uis = u0 - pb0
    seq_k0 = -uis
    nb = units_of(lens[b])
    for k in range(nu):
        while uis >= nb and b + 1 < len(lens):
            b += 1
            uis = 0
            seq_k0 = k
            nb = units_of(lens[b])
        assert uis < nb
        first = k == 0 or uis == 0
        last = k == nu - 1 or uis == nb - 1
        whole = seq_k0 >= 0 and seq_k0 + nb <= nu
        slot = 2 * c + (0 if seq_k0 <= 0 else 1)
        out.append((b, uis, first, last, whole, slot))
        uis += 1
    return out


def combine_lookup(lens, b, G):
    """The combine pass's view of row b: its CTAs cf..cl and their slots."""
    un = [units_of(x) for x in lens]
    T = sum(un)
    Pb = sum(un[:b])
    nb = un[b]
    if nb == 0:
        return None
    cf = cta_of(Pb, T, G)
    cl = cta_of(Pb + nb - 1, T, G)

    def slot_of(c):
        s0 = cta_start(c, T, G)
        return 2 * c + (0 if s0 >= Pb else 1) if s0 != cta_start(c + 1, T, G) else -1

    return cf, cl, [slot_of(c) for c in range(cf, cl + 1)]


def check(lens, G):
    loaded = {}
    written = {}  # row -> {cta: slot} of partial states
    whole = {}
    for c in range(G):
        for b, u, first, last, wh, slot in producer_walk(lens, c, G):
            assert (b, u) not in loaded, "key unit loaded twice"
            loaded[(b, u)] = c
            if last:
                if wh:
                    whole[b] = c
                else:
                    assert slot not in written.setdefault(b, {}).values()
                    written[b][c] = slot
    for b, x in enumerate(lens):
        nb = units_of(x)
        assert all((b, u) in loaded for u in range(nb)), "key unit never loaded"
        look = combine_lookup(lens, b, G)
        if nb == 0:
            assert look is None
            continue
        cf, cl, slots = look
        # CTAs between cf and cl with an empty range (T < G) wrote nothing
        # and have no slot
        held = {c: s for c, s in zip(range(cf, cl + 1), slots) if s >= 0}
        ctas = sorted({loaded[(b, u)] for u in range(nb)})
        assert ctas == sorted(held)
        if cf == cl:
            assert whole.get(b) == cf and b not in written
        else:
            assert b not in whole
            assert written[b] == held
    # two partial slots per CTA at most, and no slot shared by two rows
    seen = {}
    for b, m in written.items():
        for c, s in m.items():
            assert s // 2 == c and s not in seen
            seen[s] = b


@pytest.mark.parametrize("G", [1, 3, 148])
def test_split_producer_and_combine_agree(G):
    rng = random.Random(G)
    for trial in range(80):
        B = rng.choice([1, 2, 5, 8, 33, 128, 300])
        hi = rng.choice([16, 100, 1024, 5000])
        lens = [rng.choice([0, rng.randint(1, hi)]) if rng.random() < 0.2 else rng.randint(1, hi) for _ in range(B)]
        check(lens, G)


def test_split_edge_cases():
    G = 148
    check([0] * 7, G)                  # nothing to load
    check([1], G)                      # one unit, T < G: most CTAs have empty ranges
    check([16] * 148, G)               # one unit per row and per CTA
    check([0, 17, 0, 0, 33, 0], 4)     # empty rows between
    check([16 * 148 * 4], G)           # one long row over every CTA
    check([16] * 1024, G)              # many one-unit rows


def test_planted_slot_mistake_is_caught():
    # The combine reading slot 2c + 0 for every CTA (ignoring whether the row
    # started inside the CTA's range) must be caught by the check.
    global combine_lookup
    real = combine_lookup

    def wrong(lens, b, G):
        r = real(lens, b, G)
        if r is None:
            return r
        cf, cl, slots = r
        return cf, cl, [s - (s & 1) if s >= 0 else s for s in slots]

    combine_lookup = wrong
    try:
        with pytest.raises(AssertionError):
            check([100, 300, 50, 700], 5)
    finally:
        combine_lookup = real
