"""Barrier protocol of the tile-pair attention kernel, simulated on the host.

`lvsa_attn_pair_kernel` (csrc/lvsa_attn.cu) runs three agents per CTA: the
TMA producer, the MMA issuer and two softmax classes.  They share a K ring of
SK stages, a V ring of SV stages and per-class S / P barriers, and the
producer and issuer walk the same load sequence (`pair_step`), in which a
key tile named by both query tiles at the same step is loaded once.  This
test mirrors that sequence and the waits/arrivals of each agent as counters
(a wait on phase parity is modelled as "completions >= n" plus a check that
the barrier is not already a full phase ahead, which would alias the parity)
and runs the agents under random interleavings with MMAs retiring at once.
It checks that every list pair of the shapes the tile CSR produces (equal,
prefix / superset, disjoint, unordered, one empty, different lengths)
finishes without a deadlock or a parity alias, for the ring depths the build
uses (3 + 2) and others.
"""

import random

import pytest


def pair_step(i, l0, l1, gc):
    """Loads of step i: (g0, g1, shared); mirrors pair_step() in the kernel."""
    n0, n1 = len(l0), len(l1)
    g0 = -1
    if i < n0:
        g0, gc[0] = gc[0], gc[0] + 1
    shared = i < n0 and i < n1 and l0[i] == l1[i]
    g1 = -1
    if i < n1:
        if shared:
            g1 = g0
        else:
            g1, gc[0] = gc[0], gc[0] + 1
    return g0, g1, shared


class Alias(AssertionError):
    pass


def simulate(l0, l1, SK, SV, rng):
    cnt = {}

    def c(k):
        return cnt.get(k, 0)

    def inc(k):
        cnt[k] = c(k) + 1

    def wait(key, n):
        # mbarrier parity wait for completion n (1-based): blocks while fewer
        # than n completions; more than n means the parity would alias.
        while c(key) < n:
            yield
        if c(key) != n:
            raise Alias(f"{key}: waited for phase {n}, barrier at {c(key)}")

    nmax = max(len(l0), len(l1))

    def producer():
        gc = [0]
        for i in range(nmax):
            g0, g1, sh = pair_step(i, l0, l1, gc)
            for t in range(2):
                g = g0 if t == 0 else (-1 if sh else g1)
                if g < 0:
                    continue
                if g >= SK:
                    yield from wait(("k_empty", g % SK), g // SK)
                inc(("k_full", g % SK))
                if g >= SV:
                    yield from wait(("v_empty", g % SV), g // SV)
                inc(("v_full", g % SV))

    def issuer():
        nc = (len(l0), len(l1))

        def issue_s(cl, g, last):
            yield from wait(("k_full", g % SK), g // SK + 1)
            inc(("s_full", cl))
            if last:
                inc(("k_empty", g % SK))

        def issue_pv(cl, i, g, last):
            yield from wait(("p_full", cl), i + 1)
            yield from wait(("v_full", g % SV), g // SV + 1)
            if last:
                inc(("v_empty", g % SV))

        gc = [0]
        cur = pair_step(0, l0, l1, gc)
        if cur[0] >= 0:
            yield from issue_s(0, cur[0], not cur[2])
        if cur[1] >= 0:
            yield from issue_s(1, cur[1], True)
        for i in range(nmax):
            nxt = pair_step(i + 1, l0, l1, gc) if i + 1 < nmax else (-1, -1, False)
            for cl in range(2):
                if i >= nc[cl]:
                    continue
                yield from issue_pv(cl, i, cur[cl], cl == 1 or not cur[2])
                if i + 1 < nc[cl]:
                    yield from issue_s(cl, nxt[cl], cl == 1 or not nxt[2])
            cur = nxt
        inc("o_done")

    def softmax(cl, n):
        for it in range(n):
            yield from wait(("s_full", cl), it + 1)
            inc(("p_full", cl))

    agents = [producer(), issuer(), softmax(0, len(l0)), softmax(1, len(l1))]
    stalled = 0
    while agents:
        rng.shuffle(agents)
        progressed = False
        for a in list(agents):
            before = dict(cnt)
            try:
                next(a)
            except StopIteration:
                agents.remove(a)
                progressed = True
                continue
            progressed |= cnt != before
        stalled = 0 if progressed else stalled + 1
        if stalled > 64:
            return False
    return c("o_done") == 1


def list_pairs(rng, n):
    for _ in range(n):
        base = sorted(rng.sample(range(48), rng.randint(0, 14)))
        l0, l1 = list(base), list(base)
        r = rng.random()
        if r < 0.3:
            l1 = sorted(set(base) | set(rng.sample(range(48), rng.randint(1, 4))))
        elif r < 0.45:
            l1 = rng.sample(range(48), rng.randint(0, 14))
        elif r < 0.55:
            l1 = []
        elif r < 0.65:
            l1 = base[: rng.randint(0, len(base))]
        if rng.random() < 0.5:
            l0, l1 = l1, l0
        yield l0, l1


@pytest.mark.parametrize("SK,SV", [(3, 2), (2, 2), (2, 3), (4, 2), (6, 6), (3, 1)])
def test_pair_protocol_never_deadlocks_or_aliases(SK, SV):
    rng = random.Random(SK * 100 + SV)
    fixed = [([0, 1, 2], [0, 1, 2]), ([3, 4], [3, 4, 5, 6]), ([8, 0], [1, 7]), ([], [2, 5, 8, 1, 0, 3, 4]),
             ([6, 2, 4], []), ([], []), ([5], [5])]
    for l0, l1 in fixed + list(list_pairs(rng, 300)):
        for _ in range(3):
            assert simulate(l0, l1, SK, SV, rng), f"deadlock: SK={SK} SV={SV} lists {l0} / {l1}"


def test_shared_steps_load_once():
    gc = [0]
    steps = [pair_step(i, [0, 1, 2, 9], [0, 1, 3], gc) for i in range(4)]
    assert [s[2] for s in steps] == [True, True, False, False]
    assert gc[0] == 5  # tiles 0 and 1 shared, 2 and 3 loaded apart, 9 alone
