"""Host-side model of the barrier protocol of the batched W4A8 GEMM kernel
(ulir-kernels_b200/csrc/ks_gemm_w4a8.cu), checked under random interleavings.

The kernel's roles -- the TMA producer, eight unpack warps in two sets, one or
two MMA issuers, eight epilogue warps -- hand ring stages, tensor-memory A
slots and accumulator units to one another through mbarriers.  A parity wait
on an mbarrier is only sound while the barrier is at most one phase ahead of
or behind the waiter, so the protocol gives every barrier one waiting role
that takes its phases in order: two MMA issuers each own their accumulator
units, a hand-off whose units need more than half of them gets one issuer,
and the A slots split by hand-off parity.  This model restates the kernel's
index arithmetic and waits (shape constants as in the kernel's Shape), steps
the roles in random order, and asserts at every access that each buffer holds
what its reader expects and is overwritten only after its readers are done;
a run in which no role can move is a deadlock.  The planted mistake -- two
issuers sharing one ring of accumulator units, the kernel's earlier form,
which gave wrong results at M = 64 on the GPU -- must be caught.
"""

import random

import pytest

PROG = [0]  # arrivals so far, across all barriers: a run with none for long is stuck


class Bar:
    """An mbarrier: `count` arrivals complete a phase; done(parity) is the
    hardware's parity test (true while the current phase's parity differs)."""
    def __init__(s, count): s.count, s.pending, s.phase = count, count, 0
    def arrive(s):
        PROG[0] += 1
        s.pending -= 1
        assert s.pending >= 0
        if s.pending == 0: s.phase += 1; s.pending = s.count
    def done(s, parity): return (s.phase & 1) != parity



class Ring:
    """A ring position kept incrementally, as in the kernel."""
    def __init__(s): s.i, s.ph = 0, 0
    def next(s, n):
        s.i += 1
        if s.i == n: s.i, s.ph = 0, s.ph ^ 1
    def copy(s):
        r = Ring(); r.i, r.ph = s.i, s.ph; return r



def shape(MPAD, KPG, NA_k, PK=False):
    """The kernel's compile-time hand-off shape for Mpad tokens and G = 32 * KPG
    (PK: at most 8 tokens, two groups per 16 accumulator columns)."""
    GPS = 4 // KPG; HB = 4 if PK else 2 if GPS * MPAD <= 64 else 1; GPH = HB * GPS
    GCOLS = 8 if PK else MPAD
    UPH = 1 if GPH * GCOLS <= 192 else 2; UG = GPH // UPH; UCOLS = UG * GCOLS
    NA = NA_k if (512 - NA_k * 32) // UCOLS >= 2 else 4
    NAS = NA // HB; NACC = min(8, (512 - NA * 32) // UCOLS)
    SPLIT = MPAD == 16 and HB >= 2  # both issuers take every hand-off, half of its blocks each, one ring of units
    ISS = 2 if SPLIT or (NACC >= 2 * UPH and NAS % 2 == 0) else 1
    NPI = NACC if SPLIT else NACC // ISS  # units per ring
    return dict(GPS=GPS, HB=HB, UPH=UPH, NA=NA, NAS=NAS, NACC=NACC, ISS=ISS, NPI=NPI, SPLIT=SPLIT)



def run(MPAD=64, KPG=1, nkb=32, nst=3, NA_k=8, seed=0, shared_ring=False, PK=False):
    """One CTA over nkb 128-K blocks with an nst-stage ring; roles as
    generators that yield while they wait, stepped in random order."""
    S = shape(MPAD, KPG, NA_k, PK)
    HB, UPH, NAS, ISS, NPI = S['HB'], S['UPH'], S['NAS'], S['ISS'], S['NPI']
    SPLIT = S['SPLIT']
    if shared_ring:  # the unsound form: two issuers waiting on one ring of units
        ISS, NPI = 2, S['NACC']
    kMD = 16; kSB = 4
    nks = (nkb + kSB - 1) // kSB; nh = (nkb + HB - 1) // HB
    full = [Bar(1) for _ in range(nst)]; empty = [Bar(8 + ISS) for _ in range(nst)]
    afull = [Bar(8 if HB >= 2 else 4) for _ in range(NAS)]; mdone = [Bar(2 if SPLIT else 1) for _ in range(kMD)]
    halves = {}  # SPLIT: issuers done with a hand-off's MMAs
    nslots = NPI if (shared_ring or SPLIT) else ISS * NPI
    accempty = [Bar(8) for _ in range(nslots)]
    stage_ver = [-1] * nst; aslot = [None] * NAS; acc = [None] * nslots
    def blocks_of(ks): return min(kSB, nkb - ks * kSB)
    def wait(bar, parity):
        while not bar.done(parity): yield
    def producer():
        for ks in range(nks):
            s = ks % nst
            if ks >= nst: yield from wait(empty[s], ((ks // nst) - 1) & 1)
            stage_ver[s] = ks
            yield
            full[s].arrive()
    def unpack(set_, q):
        for ks in range(nks):
            s = ks % nst
            yield from wait(full[s], (ks // nst) & 1)
            assert stage_ver[s] == ks
            nb = blocks_of(ks)
            j0 = 0 if HB >= 2 else set_
            while j0 < nb:
                h = (ks * kSB + j0) // HB; slot = h % NAS
                if h >= NAS: yield from wait(mdone[(h - NAS) % kMD], ((h - NAS) // kMD) & 1)
                # this warp's blocks of the hand-off: j0 + set, j0 + set + 2, ... (HB >= 2)
                for jj in (range(set_, HB, 2) if HB >= 2 else (0,)):
                    j = j0 + jj
                    if j < nb:
                        if q == 0:
                            assert aslot[slot] is None or aslot[slot][1] == 'read' or aslot[slot][0] == h, ("A overwrite", h, aslot[slot])
                            aslot[slot] = (h, 'writing')
                        yield
                        assert stage_ver[s] == ks
                afull[slot].arrive()
                j0 += HB if HB >= 2 else 2
            empty[s].arrive()
    def mma(mine):
        if mine >= ISS: return
        st, asr, ac = Ring(), Ring(), Ring()  # ac: this issuer's own unit ring
        j0 = 0
        for h in range(nh):
            issue = SPLIT or (h % ISS) == mine
            if issue:
                yield from wait(full[st.i], st.ph)
                yield from wait(afull[asr.i], asr.ph)
                if shared_ring:
                    ac = Ring(); [ac.next(NPI) for _ in range(h * UPH)]
                u = ac.copy(); k0 = (h * UPH) if (shared_ring or SPLIT) else (h // ISS) * UPH
                base = 0 if (shared_ring or SPLIT) else mine * NPI
                for k in range(UPH):
                    if k0 + k >= NPI: yield from wait(accempty[base + u.i], u.ph ^ 1)
                    u.next(NPI)
                a = aslot[asr.i]
                assert a is not None and a[0] == h and a[1] == 'writing', ("MMA reads wrong A", h, a)
                u = ac.copy()
                for k in range(UPH):
                    sl = base + u.i
                    ok_prev = acc[sl] is None or acc[sl][2] == 'read' or (SPLIT and acc[sl][0] == h)
                    assert ok_prev, ("acc overwrite", h, acc[sl])
                    acc[sl] = (h, k, 'computing', 0); u.next(NPI)
                assert stage_ver[st.i] == (h * HB) // kSB
                yield
                n_done = halves.get(h, 0) + 1
                halves[h] = n_done
                if not SPLIT or n_done == 2:  # both halves of the hand-off issued and complete
                    aslot[asr.i] = (h, 'read')
                    u = ac.copy()
                    for k in range(UPH):
                        sl = base + u.i; acc[sl] = (h, k, 'ready', 0); u.next(NPI)
                for k in range(UPH): ac.next(NPI)
                mdone[h % kMD].arrive()
            asr.next(NAS)
            j0 += HB
            if j0 == kSB or h == nh - 1:
                empty[st.i].arrive(); st.next(nst); j0 = 0
    def epilogue(w):
        rings = [Ring() for _ in range(ISS)]
        for h in range(nh):
            yield from wait(mdone[h % kMD], (h // kMD) & 1)
            i = 0 if (shared_ring or SPLIT) else h % ISS
            for u in range(UPH):
                sl = i * NPI + rings[i].i
                a = acc[sl]
                assert a is not None and a[0] == h and a[1] == u and a[2] == 'ready', ("epilogue reads", h, u, a, w)
                yield
                a = acc[sl]; assert a[0] == h and a[1] == u and a[2] == 'ready'
                n = a[3] + 1
                acc[sl] = (h, u, 'read' if n == 8 else 'ready', n)
                accempty[sl].arrive()
                rings[i].next(NPI)
    rng = random.Random(seed)
    roles = [producer()] + [unpack(s_, q) for s_ in (0, 1) for q in range(4)] + [mma(0), mma(1)] + [epilogue(w) for w in range(8)]
    alive = list(roles); idle = 0; last = PROG[0]
    while alive:
        r = rng.choice(alive)
        try: next(r)
        except StopIteration: alive.remove(r); idle = 0
        if PROG[0] != last: last = PROG[0]; idle = 0
        else: idle += 1
        if idle > 5000 * len(alive): raise RuntimeError("deadlock")
    return S



SHAPES = [(m, k, na, False) for m in (16, 32, 48, 64) for k in (1, 2, 4) for na in (4, 8)] + \
    [(16, k, na, True) for k in (1, 2, 4) for na in (4, 8)]


@pytest.mark.parametrize("mpad,kpg,na,pk", SHAPES)
def test_protocol_hands_every_buffer_over_in_order(mpad, kpg, na, pk):
    for nkb in (1, 2, 3, 5, 33):
        for nst in (2, 3, 5):
            for seed in range(3):
                run(MPAD=mpad, KPG=kpg, NA_k=na, nkb=nkb, nst=nst, seed=seed, PK=pk)


def test_shared_accumulator_ring_is_caught():
    """Two issuers waiting on one ring of units (M = 64: two units per
    hand-off, two units in all): some interleaving reuses a unit the epilogue
    has not read, or leaves a waiter two phases behind."""
    caught = 0
    for seed in range(20):
        try:
            run(MPAD=64, KPG=1, NA_k=8, nkb=32, nst=3, seed=seed, shared_ring=True)
        except (AssertionError, RuntimeError):
            caught += 1
    assert caught > 0


def test_issuer_count_per_shape():
    """One issuer exactly where a hand-off's units need more than half of them."""
    assert shape(16, 1, 8)["ISS"] == 2 and shape(16, 1, 8)["SPLIT"] and shape(16, 1, 8)["NPI"] == 2
    assert shape(32, 2, 8)["ISS"] == 2 and not shape(32, 2, 8)["SPLIT"] and shape(32, 2, 8)["NPI"] == 1
    assert shape(16, 1, 8, PK=True)["ISS"] == 2 and shape(16, 1, 8, PK=True)["HB"] == 4
    assert shape(64, 1, 8)["ISS"] == 1 and shape(64, 1, 8)["UPH"] == 2
    for m in (16, 32, 48, 64):
        for k in (1, 2, 4):
            s = shape(m, k, 8)
            assert s["NPI"] >= s["UPH"] and s["NACC"] >= 2 and (s["ISS"] == 1 or s["NAS"] % 2 == 0)
