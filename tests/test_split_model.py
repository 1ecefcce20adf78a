"""
CPU model of the balanced K split's index arithmetic in the block-scaled GEMM (BsSegs in
lazylora_b200/csrc/bs_gemm.cuh), checked over many launch shapes: with n_units units of n_stage
K stages shared out over G CTAs in contiguous ranges [b tot / G, (b+1) tot / G), every stage is
run by exactly one CTA; every partial piece of a unit writes its own slot (2 per CTA: its first
piece, or a later one); and the finishing CTA's view of a unit (b0 = owner of its first stage,
nseg = owner of its last - b0 + 1, slot(o) = 2 (b0 + o) + [o == 0 and b0's range starts before
the unit]) names exactly the slots its pieces wrote, in CTA order. The kernel enables the split
only for n_units >= G, which keeps every range non-empty. The model restates the kernel's
formulas line for line; a change to one must be made to the other.
"""
import random


def _segs(b, G, nu, ns):
    tot = nu * ns
    g, end = tot * b // G, tot * (b + 1) // G
    first, out = True, []
    while g < end:
        u = g // ns
        u0, u1 = u * ns, u * ns + ns
        out.append((u, g - u0, min(u1, end) - u0, 0 if first else 1))
        first = False
        g = u1
    return out


def _check(nu, ns, G):
    tot = nu * ns
    begin = lambda b: tot * b // G
    owner = lambda gs: ((gs + 1) * G - 1) // tot
    cover, writers = {}, {}
    for b in range(G):
        segs = _segs(b, G, nu, ns)
        assert segs, (nu, ns, G, b)
        for u, k0, k1, piece in segs:
            for ks in range(k0, k1):
                assert (u, ks) not in cover
                cover[(u, ks)] = b
            if not (k0 == 0 and k1 == ns):
                writers.setdefault(u, []).append((b, 2 * b + piece))
    assert len(cover) == tot
    slots = [s for w in writers.values() for _, s in w]
    assert len(slots) == len(set(slots)) and max(slots, default=0) < 2 * G
    for u, w in writers.items():
        us = u * ns
        b0 = owner(us)
        nseg = owner(us + ns - 1) - b0 + 1
        want = [2 * (b0 + o) + (1 if (o == 0 and begin(b0) < us) else 0) for o in range(nseg)]
        assert [s for _, s in sorted(w)] == want, (u, want, w)
        assert [b for b, _ in sorted(w)] == list(range(b0, b0 + nseg))


def test_split_model_decode_shapes():
    # configs[3]'s F1 / F2 unit counts (T = 1, 4, 16) on 148 CTAs, and edge cases
    for nu, ns in [(128 * 2, 56), (352, 56), (224, 16), (616, 16), (1152, 56), (148, 16), (149, 1), (296, 8),
                   (1280, 56), (148, 1)]:
        _check(nu, ns, 148)


def test_split_model_random_shapes():
    rnd = random.Random(1)
    for _ in range(2000):
        G = rnd.randint(1, 160)
        ns = rnd.randint(1, 64)
        nu = rnd.randint(G, 1280 if G <= 1280 else G)
        _check(nu, ns, G)
