"""Race and deadlock check of the attention kernel's mbarrier protocol (csrc/bsa_attn.cu), on the CPU.

The kernel's roles (Q+K producer, V producer, QK issuer, PV issuer, 8 softmax warps) are restated as
sequences of waits and arrivals on the same barriers, with the same phase arithmetic.  Asynchronous
completions (TMA loads, tcgen05.commit after an MMA group) arrive later at random times, in issue
order per issuing thread.  A random scheduler runs the roles to completion and checks, at every wait,
the property the hardware needs: a parity wait for phase p must see the barrier at phase p or p + 1
(`mbarrier.try_wait.parity` only distinguishes even from odd phases, so a barrier two phases ahead of
a waiter, or a waiter one phase ahead of its barrier, would be misread).  It also checks that no
schedule deadlocks.

The GPU parity tests run many units per CTA only at k = 85; this covers the other step counts (k = 1
and 2 leave lane half 1 idle), ring sizes and unit counts per CTA in seconds.
"""
import random

import pytest


class Barrier:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.completed = 0   # completed phases
        self.pending = 0     # arrivals in the current phase

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending = 0
            self.completed += 1


class AliasError(AssertionError):
    pass


def wait(bar, phase):
    """A role waits for `phase` of `bar` to complete.  Returns True when it may proceed.

    The hardware wait sees only the parity of the barrier's current phase, so it reads correctly only
    while the barrier has completed `phase` or `phase + 1` phases.  Two more (the barrier ran a whole
    phase past the waiter) or one fewer (the waiter is a phase ahead: the previous phase of the same
    parity would read as complete) are both misreads."""
    if bar.completed >= phase + 2 or bar.completed < phase:
        raise AliasError(f"{bar.name}: waiter for phase {phase} sees {bar.completed} completed phases")
    return bar.completed == phase + 1


def run_protocol(units, nsteps, kstages, vslots, qbufs, seed, rescale_prob=0.2):
    rng = random.Random(seed)
    two_halves = nsteps >= 2
    copy_warps = 8 if two_halves else 4
    B = {}

    def bar(name, count=1):
        B[name] = Barrier(name, count)

    for s in range(kstages):
        bar(("k_full", s)); bar(("k_empty", s))
    for s in range(vslots):
        bar(("v_full", s)); bar(("v_empty", s))
    for h in range(2):
        bar(("s_full", h)); bar(("s_empty", h), 4); bar(("q_ready", h), 4)
        for b in range(2):
            bar(("p_full", h, b), 4); bar(("p_empty", h, b))
    for b in range(qbufs):
        bar(("q_full", b)); bar(("q_empty", b), copy_warps)
    for q in range(4):
        bar(("ep", q), 2)
    bar(("o_empty",), 8)

    # asynchronous completions, per issuing thread: tcgen05.commit arrivals complete in issue order
    # (a commit tracks every earlier MMA of its thread); TMA loads may complete in any order
    async_q = {"tma_k": [], "tma_v": [], "tma_q": [], "mma_qk": [], "mma_pv": []}
    in_order = {"mma_qk", "mma_pv"}

    hs = ((nsteps + 1) // 2, nsteps // 2)

    def producer_qk():
        g = 0
        for n in range(units):
            qb = n % qbufs
            if n >= qbufs:
                while not wait(B[("q_empty", qb)], (n - qbufs) // qbufs):
                    yield
            async_q["tma_q"].append(("q_full", qb))
            for j in range(nsteps):
                ks = g % kstages
                if g >= kstages:
                    while not wait(B[("k_empty", ks)], g // kstages - 1):
                        yield
                async_q["tma_k"].append(("k_full", ks))
                g += 1
                yield

    def producer_v():
        gb = 0
        for n in range(units):
            for j in range(nsteps):
                for _ in range(2):
                    vs = gb % vslots
                    if gb >= vslots:
                        while not wait(B[("v_empty", vs)], gb // vslots - 1):
                            yield
                    async_q["tma_v"].append(("v_full", vs))
                    gb += 1
                    yield

    def issuer_qk():
        g, cnt = 0, [0, 0]
        for n in range(units):
            for j in range(nsteps):
                h = j & 1
                i = cnt[h]
                while not wait(B[("k_full", g % kstages)], g // kstages):
                    yield
                if i >= 1:
                    while not wait(B[("s_empty", h)], i - 1):
                        yield
                if j == h:
                    while not wait(B[("q_ready", h)], n):
                        yield
                async_q["mma_qk"].append(("s_full", h))
                async_q["mma_qk"].append(("k_empty", g % kstages))
                cnt[h] += 1
                g += 1
                yield

    def issuer_pv():
        g, cnt = 0, [0, 0]
        for n in range(units):
            for j in range(nsteps):
                h = j & 1
                i = cnt[h]
                for bi in range(2):
                    gb = 2 * g + bi
                    while not wait(B[("v_full", gb % vslots)], gb // vslots):
                        yield
                while not wait(B[("p_full", h, i & 1)], i >> 1):
                    yield
                if j == 0 and n >= 1:
                    while not wait(B[("o_empty",)], n - 1):
                        yield
                async_q["mma_pv"].append(("v_empty", (2 * g) % vslots))
                async_q["mma_pv"].append(("v_empty", (2 * g + 1) % vslots))
                async_q["mma_pv"].append(("p_empty", h, i & 1))
                cnt[h] += 1
                g += 1
                yield

    def softmax(h, qq):
        active = h == 0 or two_halves
        i = 0

        def copy_q(nn):
            qb = nn % qbufs
            while not wait(B[("q_full", qb)], nn // qbufs):
                yield
            B[("q_ready", h)].arrive()
            B[("q_empty", qb)].arrive()

        if active and units > 0:
            yield from copy_q(0)
        for n in range(units):
            if active:
                for s in range(hs[h]):
                    while not wait(B[("s_full", h)], i):
                        yield
                    B[("s_empty", h)].arrive()
                    yield
                    if s > 0 and rng.random() < rescale_prob:  # the lazy max moved: O of this half is rescaled
                        while not wait(B[("p_empty", h, (i - 1) & 1)], (i - 1) >> 1):
                            yield
                    if i >= 2:
                        while not wait(B[("p_empty", h, i & 1)], (i - 2) >> 1):
                            yield
                    B[("p_full", h, i & 1)].arrive()
                    i += 1
                    yield
                if n + 1 < units:
                    yield from copy_q(n + 1)
            if active:  # this half's last PV of the unit; the ep handshake carries the other half's
                last = i - 1
                while not wait(B[("p_empty", h, last & 1)], last >> 1):
                    yield
            B[("ep", qq)].arrive()
            while not wait(B[("ep", qq)], n):
                yield
            # O is read here: every PV of this unit, in both halves, must have completed
            for hh in ((0, 1) if two_halves else (0,)):
                lh = (n + 1) * hs[hh] - 1
                assert B[("p_empty", hh, lh & 1)].completed >= (lh >> 1) + 1, ("O read early", n, hh)
            B[("o_empty",)].arrive()
            yield

    roles = [producer_qk(), producer_v(), issuer_qk(), issuer_pv()] + [softmax(h, q) for h in (0, 1) for q in range(4)]
    live = list(range(len(roles)))
    stalls = 0
    while live or any(async_q.values()):
        # either complete one pending asynchronous operation, or step one role
        pending = [k for k, v in async_q.items() if v]
        if pending and (not live or rng.random() < 0.35):
            k = rng.choice(pending)
            B[async_q[k].pop(0 if k in in_order else rng.randrange(len(async_q[k])))].arrive()
            stalls = 0
            continue
        r = rng.choice(live)
        before = tuple((b.completed, b.pending) for b in B.values())
        try:
            next(roles[r])
        except StopIteration:
            live.remove(r)
            stalls = 0
            continue
        after = tuple((b.completed, b.pending) for b in B.values())
        stalls = stalls + 1 if before == after and not pending else 0
        if stalls > 5000:
            raise AssertionError(f"deadlock: units={units} nsteps={nsteps} rings=({kstages},{vslots},{qbufs})")
    # every phase of every barrier ran to completion: no arrival is left over
    assert all(b.pending == 0 for b in B.values()), [b.name for b in B.values() if b.pending]


@pytest.mark.parametrize("nsteps", [1, 2, 3, 4, 43])
@pytest.mark.parametrize("units", [1, 2, 5])
@pytest.mark.parametrize("rings", [(2, 8, 2), (3, 6, 2), (2, 9, 1), (4, 4, 2)])
def test_attention_barrier_protocol(nsteps, units, rings):
    for seed in range(6 if nsteps < 43 else 2):
        run_protocol(units, nsteps, *rings, seed=seed)


def test_protocol_model_detects_aliasing():
    """The checker is live: a waiter that lags its barrier by two phases, or runs a phase ahead of it,
    is reported."""
    b = Barrier("x", 1)
    b.arrive(); b.arrive()
    with pytest.raises(AliasError):
        wait(b, 0)
    with pytest.raises(AliasError):
        wait(Barrier("y", 1), 1)


# ------------------------------------------------------------------ the pooling kernel's TMA ring
def run_pool_ring(cnt, consumers, ring, owned, seed, p_land=0.1):
    """csrc/bsa_score.cu pool_tma_kernel: one producer lane streams `cnt` blocks into `ring` slots; each
    block is reduced by one of `consumers` warps.  owned=True is the kernel's layout (consumer c takes
    blocks c, c + consumers, ... into its own two slots); owned=False is a shared ring with round-robin
    blocks.  TMA loads complete in any order."""
    rng = random.Random(seed)
    full = [Barrier(("full", s), 1) for s in range(ring)]
    empty = [Barrier(("empty", s), 1) for s in range(ring)]
    per = ring // consumers

    def place(i):
        if owned:
            m = i // consumers
            return (i % consumers) * per + (m % per), m // per
        return i % ring, i // ring

    tma = []

    def producer():
        for i in range(cnt):
            slot, fill = place(i)
            if fill >= 1:
                while not wait(empty[slot], fill - 1):
                    yield
            tma.append(slot)
            yield

    def consumer(c):
        for i in range(c, cnt, consumers):
            slot, fill = place(i)
            while not wait(full[slot], fill):
                yield
            yield  # rows read into registers
            empty[slot].arrive()

    roles = [producer()] + [consumer(c) for c in range(consumers)]
    live = list(range(len(roles)))
    stalls = 0
    while live or tma:
        if tma and (not live or rng.random() < p_land):
            full[tma.pop(rng.randrange(len(tma)))].arrive()
            continue
        r = rng.choice(live)
        try:
            next(roles[r])
            stalls += 1
        except StopIteration:
            live.remove(r)
            stalls = 0
        if stalls > 200000:
            raise AssertionError("deadlock")
    assert all(b.pending == 0 for b in full + empty)


@pytest.mark.parametrize("cnt", [1, 5, 12, 13, 97, 292])
def test_pool_ring_protocol(cnt):
    for seed in range(8):
        run_pool_ring(cnt, consumers=6, ring=12, owned=True, seed=seed)


def test_pool_ring_model_rejects_shared_round_robin_ring():
    """The layout the kernel replaced (8 warps round-robin over a shared 12-slot ring) lets a consumer
    wait on a slot whose previous block has not landed yet; the model reports it."""
    with pytest.raises(AliasError):
        for seed in range(50):
            run_pool_ring(292, consumers=8, ring=12, owned=False, seed=seed)
