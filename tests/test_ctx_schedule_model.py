"""The fused step's context phase (k_step.cu, attn_ctx_ring and Producer::ctx_slots) as a
protocol model on the CPU: the producer, the four helper warps and the chain warp of one
CTA run as coroutines under random interleavings, over mbarriers with the hardware's
phase-parity semantics. Every interleaving must finish (no deadlock), the chain must read
each block's products in order and never a buffer a helper is rewriting, and no V copy
may land in a ring slot before its previous block was read. The item map (`ctx_item`)
must give every (query head, slice) item to exactly one CTA, for more and for fewer
items than CTAs."""
import random

import pytest

HELPERS = 4          # kCtxHelpers: helper warps 1, 2, 3, 5, one products buffer each
CONS_WARPS = 8       # kConsWarps: the empty barrier's arrival count


class MBar:
    """mbarrier: `count` arrivals complete the current phase; test_wait.parity(p) is true
    once the phase of parity p has completed (for a fresh barrier, parity 1 counts as
    completed: the phase before phase 0)."""

    def __init__(self, count):
        self.count, self.arrived, self.phase = count, 0, 0

    def arrive(self, n=1):
        self.arrived += n
        assert self.arrived <= self.count, "more arrivals than the phase expects"
        if self.arrived == self.count:
            self.arrived, self.phase = 0, self.phase + 1

    def done(self, parity):
        return (self.phase & 1) != parity


class Wait(Exception):
    pass


def ctx_item(b, grid, nitems, j):
    """k_step.cu ctx_item."""
    if nitems > grid:
        k = j * grid + b
        return k if k < nitems else -1
    if j > 0:
        return -1
    k = (b * nitems + grid - 1) // grid
    return k if k < nitems and (k * grid) // nitems == b else -1


def simulate(nblks, ns, seed):
    """One CTA's phase B over consecutive items with nblks[i] blocks each (the ring has
    ns slots and starts at sequence number 0). Returns the number of scheduling steps."""
    rng = random.Random(seed)
    full = [MBar(1) for _ in range(ns)]
    empty = [MBar(CONS_WARPS) for _ in range(ns)]
    pfull = [MBar(1) for _ in range(HELPERS)]
    pfree = [MBar(1) for _ in range(HELPERS)]
    slot = [None] * ns              # which block's V rows a slot holds
    pbuf = [None] * HELPERS         # which block's products a buffer holds
    readers = [0] * HELPERS         # chain reads in progress per buffer (half blocks)
    log = []

    def producer():
        q = 0
        for nb in nblks:
            for k in range(nb):
                s = q % ns
                while not (q < ns or empty[s].done(((q // ns) & 1) ^ 1)):
                    yield
                # the previous block in this slot must be fully read by its helper
                assert slot[s] is None or slot[s][1] == "read", ("V overwrite", q)
                slot[s] = ((q, k), "landed")
                full[s].arrive()
                q += 1
                yield

    def helper(h):
        q0 = u0 = 0
        for nb in nblks:
            kfirst = (h + HELPERS - u0 % HELPERS) % HELPERS
            for k in range(kfirst, nb, HELPERS):
                q, u = q0 + k, u0 + k
                c = u // HELPERS
                s = q % ns
                while not full[s].done((q // ns) & 1):
                    yield
                assert slot[s] == ((q, k), "landed"), ("helper reads a wrong slot", slot[s], q)
                slot[s] = ((q, k), "read")
                empty[s].arrive(CONS_WARPS // 1)        # one arrive with the whole count
                yield
                if c > 0:
                    while not pfree[h].done((c - 1) & 1):
                        yield
                assert readers[h] == 0, "helper rewrites a buffer the chain is reading"
                pbuf[h] = u
                yield
                pfull[h].arrive()
                yield
            q0 += nb
            u0 += nb

    def chain():
        u0 = 0
        for nb in nblks:
            def wait_blk(k):
                u = u0 + k
                b = u % HELPERS
                while not pfull[b].done((u // HELPERS) & 1):
                    yield
                assert pbuf[b] == u, ("chain reads a wrong buffer", pbuf[b], u)

            def read_half(k):
                b = (u0 + k) % HELPERS
                assert pbuf[b] == u0 + k
                readers[b] += 1
                yield
                readers[b] -= 1

            yield from wait_blk(0)
            yield from read_half(0)
            yield from read_half(0)
            for k in range(nb):
                log.append(u0 + k)                  # the adds of block k
                more = k + 1 < nb
                if more:
                    yield from wait_blk(k + 1)
                    yield from read_half(k + 1)
                yield
                if more:
                    yield from read_half(k + 1)
                pfree[(u0 + k) % HELPERS].arrive()
                yield
            u0 += nb

    actors = [producer(), chain()] + [helper(h) for h in range(HELPERS)]
    live = list(actors)
    steps = 0
    stuck = 0
    while live:
        a = rng.choice(live)
        before = (tuple(m.phase for m in full + empty + pfull + pfree), tuple(slot),
                  tuple(pbuf), len(log))
        try:
            next(a)
        except StopIteration:
            live.remove(a)
            stuck = 0
            continue
        steps += 1
        after = (tuple(m.phase for m in full + empty + pfull + pfree), tuple(slot),
                 tuple(pbuf), len(log))
        stuck = 0 if after != before else stuck + 1
        assert stuck < 20000, "no actor can make progress: deadlock"
    assert log == list(range(sum(nblks))), "the chain added blocks out of order"
    return steps


@pytest.mark.parametrize("nblks", [[1], [2], [5], [9, 9], [3, 7], [1, 1, 1], [66]])
@pytest.mark.parametrize("ns", [5, 15])
def test_context_phase_protocol(nblks, ns):
    for seed in range(12):
        simulate(nblks, ns, seed)


@pytest.mark.parametrize("grid,nitems", [(148, 128), (148, 256), (148, 64), (148, 32),
                                         (132, 256), (148, 148), (148, 600)])
def test_ctx_item_covers_every_item_once(grid, nitems):
    seen = []
    for b in range(grid):
        j = 0
        while (it := ctx_item(b, grid, nitems, j)) >= 0:
            seen.append(it)
            j += 1
    assert sorted(seen) == list(range(nitems))
