"""A CPU model of the W4A16 pair kernel's barrier protocol (gemm_w4a16_pair_kernel in
csrc/nvfp4_w4a16.cu), run under random schedules.

Two CTAs (rank 0 leads) walk the pair's tiles.  Per CTA, a producer fills a ring of `stages`
slots (full[s]: its activation, packed-weight and scale loads landed, completing in any order
across slots); the converter warps -- `groups` groups of four per CTA, group g taking the stages
it with it % groups == g -- wait for full[s], write the slot's widened weight tile and arrive at
the leader's ready[s] (8 arrivals: one group of each CTA); the leader's MMA thread waits for
ready[s], reads both CTAs' slot s, and commits empty[s] of both CTAs (commits complete in issue
order) and, after a tile, accf[b] of both CTAs for accumulator b = tile % 2; the eight epilogue
warps of each CTA wait for accf[b], drain it and arrive at the leader's acce[b] (16 arrivals),
which the MMA thread waits for before it reuses accumulator b.

Checks: every run ends (no deadlock), no parity wait is more than one phase behind, no slot is
refilled or re-widened before the MMA read it, the MMA reads only slots whose loads and both
CTAs' widening belong to its own K step, and no accumulator is overwritten before all sixteen
epilogue warps drained it."""
import random

import pytest


class Bar:
    def __init__(self, count=1):
        self.count, self.pending, self.done = count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.done += 1
            self.pending = self.count


def run(tiles, nks, stages, groups, seed):
    rnd = random.Random(seed)
    full = [[Bar() for _ in range(stages)] for _ in range(2)]
    empty = [[Bar() for _ in range(stages)] for _ in range(2)]
    ready = [Bar(8) for _ in range(stages)]                      # leader's
    accf = [[Bar(), Bar()] for _ in range(2)]
    acce = [Bar(16), Bar(16)]                                    # leader's
    loaded = [[None] * stages for _ in range(2)]                 # K step whose loads landed in the slot
    widened = [[dict() for _ in range(stages)] for _ in range(2)]  # K step -> warps that widened it
    consumed = [[True] * stages for _ in range(2)]               # the MMA read the slot's last use
    acc = [None, None]                                           # (tile, drained warps)
    tick = [0]
    loads, commits = [], []                                      # pending async completions
    total = tiles * nks

    def later(fn):
        loads.append((tick[0] + rnd.randint(1, 6), fn))           # TMA: any order across slots

    def commit(fn):
        t = tick[0] + rnd.randint(1, 4)
        if commits:
            t = max(t, commits[-1][0])                           # tcgen05.commit: in issue order
        commits.append((t, fn))

    def wait(b, phase):
        while b.done <= phase:
            yield
        assert b.done <= phase + 1, "parity alias: the barrier ran a phase ahead of this wait"

    def producer(r):
        for it in range(total):
            s = it % stages
            if it >= stages:
                yield from wait(empty[r][s], it // stages - 1)
            assert consumed[r][s], "slot refilled before the MMA read it"
            consumed[r][s] = False

            def land(r=r, s=s, it=it):
                loaded[r][s] = it
                full[r][s].arrive()
            later(land)
            yield

    def converter(r, g, w):
        for it in range(total):
            if it % groups != g:
                continue
            s = it % stages
            yield from wait(full[r][s], it // stages)
            assert loaded[r][s] == it
            assert not consumed[r][s], "widening a slot the MMA already read"
            yield
            widened[r][s].setdefault(it, set()).add(w)
            ready[s].arrive()

    def mma():
        it = 0
        for lt in range(tiles):
            b, use = lt & 1, lt >> 1
            if use > 0:
                yield from wait(acce[b], use - 1)
            assert acc[b] is None or len(acc[b][1]) == 16, "accumulator overwritten before it was drained"
            acc[b] = (lt, set())
            for _ in range(nks):
                s = it % stages
                yield from wait(ready[s], it // stages)
                for r in range(2):
                    assert loaded[r][s] == it and len(widened[r][s].get(it, ())) == 4, "MMA read a stale slot"

                def release(s=s, it=it):
                    for r in range(2):
                        consumed[r][s] = True
                        widened[r][s].pop(it)
                        empty[r][s].arrive()
                commit(release)
                it += 1
            for r in range(2):
                commit(lambda r=r, b=b: accf[r][b].arrive())

    def epilogue(r, w):
        for lt in range(tiles):
            b, use = lt & 1, lt >> 1
            yield from wait(accf[r][b], use)
            assert acc[b][0] == lt
            yield
            acc[b][1].add((r, w))
            acce[b].arrive()

    live = [producer(0), producer(1), mma()]
    live += [converter(r, g, w) for r in range(2) for g in range(groups) for w in range(4)]
    live += [epilogue(r, w) for r in range(2) for w in range(8)]
    for _ in range(400000):
        tick[0] += 1
        for q in (loads, commits):
            due = [e for e in q if e[0] <= tick[0]]
            for e in due:
                q.remove(e)
            if q is loads:
                rnd.shuffle(due)
            for _, fn in due:
                fn()
        if not live and not loads and not commits:
            assert all(a is None or len(a[1]) == 16 for a in acc)
            return
        rnd.shuffle(live)
        for c in list(live)[: rnd.randint(1, len(live))]:
            try:
                next(c)
            except StopIteration:
                live.remove(c)
    raise AssertionError("the protocol did not finish (deadlock)")


@pytest.mark.parametrize("tiles", [1, 2, 5])
@pytest.mark.parametrize("nks,stages", [(1, 5), (4, 5), (7, 5), (9, 3)])
@pytest.mark.parametrize("groups", [1, 2, 3, 4])
def test_w4a16_pair_protocol_random_schedules(tiles, nks, stages, groups):
    for seed in range(6):
        run(tiles, nks, stages, groups, seed)
