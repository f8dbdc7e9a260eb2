"""A CPU model of the W4A4 pair GEMM's barrier protocol (gemm_pair_kernel in csrc/nvfp4_gemm.cu),
run under random schedules.

Two CTAs (rank 0 leads) walk the pair's tiles over a ring of `stages` slots.  Only the leader's
full[s] is used: its producer arms it with both CTAs' bytes (one arrival + 2 x STAGE bytes), and
both CTAs' loads complete their bytes on it, in any order and possibly before the arming.  Each
CTA's producer refills slot s only after its own empty[s], which the leader's MMA thread commits
to both CTAs once the slot is read.  The MMA thread copies each stage's scale factors into that
slot's TMEM columns before the stage's MMAs; for the first `pre` stages of a tile it does so
before waiting for the single accumulator to drain (acce, 16 arrivals: the eight epilogue warps
of both CTAs), so those copies can overlap the previous tile's epilogue.  tcgen05 copies, MMAs
and commits of that one thread execute in issue order.  After a tile's last MMA it commits accf
to both CTAs; the epilogue warps wait for it, drain the accumulator and release it.

Checks: every run ends, no parity wait is more than one phase behind, the bytes landing on the
leader's full[s] all belong to the phase being filled, no slot is refilled before the MMA read it,
the MMA reads only slots (both CTAs' data and the scale columns) of its own K step, and no tile's
MMAs start before all sixteen epilogue warps drained the previous tile."""
import random

import pytest

STAGE = 38912


class TxBar:
    """mbarrier with a transaction count: a phase completes when its arrivals are in and its
    byte count is back to zero (bytes may land before the arming arrival)."""

    def __init__(self, count=1):
        self.count, self.pending, self.tx, self.done = count, count, 0, 0

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.done += 1
            self.pending = self.count

    def arrive(self, expect=0):
        self.pending -= 1
        assert self.pending >= 0
        self.tx += expect
        self._check()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._check()


def run(tiles, nkt, stages, pre, seed):
    rnd = random.Random(seed)
    full = [TxBar() for _ in range(stages)]                         # leader's
    empty = [[TxBar() for _ in range(stages)] for _ in range(2)]
    accf = [TxBar(), TxBar()]
    acce = TxBar(16)                                                # leader's
    loaded = [[None] * stages for _ in range(2)]
    consumed = [[True] * stages for _ in range(2)]
    scales = [None] * stages                                        # K step whose scale factors sit in the slot's columns
    acc = {"tile": None, "drained": set(), "writing": None}
    tick = [0]
    loads, tc = [], []                                              # TMA completions; the tcgen05 queue (in order)
    total = tiles * nkt

    def later(fn):
        loads.append((tick[0] + rnd.randint(1, 6), fn))

    def tcgen05(fn):
        t = tick[0] + rnd.randint(1, 4)
        if tc:
            t = max(t, tc[-1][0])
        tc.append((t, fn))

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
            if r == 0:
                full[s].arrive(2 * STAGE)

            def land(r=r, s=s, it=it):
                assert full[s].done == it // stages, "bytes landed on another phase of the stage barrier"
                loaded[r][s] = it
                full[s].complete_tx(STAGE)
            later(land)
            yield

    def mma():
        it = 0

        def copy_scales(i):
            s = i % stages
            assert loaded[0][s] == i and loaded[1][s] == i

            def done(s=s, i=i):
                scales[s] = i
            tcgen05(done)

        for lt in range(tiles):
            p = min(pre, nkt)
            for j in range(p):
                yield from wait(full[(it + j) % stages], (it + j) // stages)
                copy_scales(it + j)
            if lt > 0:
                yield from wait(acce, lt - 1)
                assert acc["drained"] == {(r, w) for r in range(2) for w in range(8)}, "accumulator reused early"
            for kt in range(nkt):
                s = it % stages
                if kt >= p:
                    yield from wait(full[s], it // stages)
                    copy_scales(it)

                def mma_step(s=s, it=it, lt=lt):
                    assert loaded[0][s] == it and loaded[1][s] == it and scales[s] == it, "MMA read a stale slot"
                    if acc["tile"] != lt:
                        assert acc["tile"] is None or len(acc["drained"]) == 16, "accumulator overwritten"
                        acc["tile"], acc["drained"] = lt, set()

                def release(s=s):
                    for r in range(2):
                        consumed[r][s] = True
                        empty[r][s].arrive()
                tcgen05(mma_step)
                tcgen05(release)
                it += 1
            for r in range(2):
                tcgen05(lambda r=r: accf[r].arrive())

    def epilogue(r, w):
        for lt in range(tiles):
            yield from wait(accf[r], lt)
            assert acc["tile"] == lt
            yield
            acc["drained"].add((r, w))
            acce.arrive()
            yield  # the stores follow the release

    live = [producer(0), producer(1), mma()] + [epilogue(r, w) for r in range(2) for w in range(8)]
    for _ in range(400000):
        tick[0] += 1
        for q in (loads, tc):
            due = [e for e in q if e[0] <= tick[0]]
            for e in due:
                q.remove(e)
            if q is loads:
                rnd.shuffle(due)
            for _, fn in due:
                fn()
        if not live and not loads and not tc:
            assert len(acc["drained"]) == 16
            return
        rnd.shuffle(live)
        for c in list(live)[: rnd.randint(1, len(live))]:
            try:
                next(c)
            except StopIteration:
                live.remove(c)
    raise AssertionError("the protocol did not finish (deadlock)")


@pytest.mark.parametrize("tiles", [1, 2, 4])
@pytest.mark.parametrize("nkt,stages", [(1, 5), (2, 5), (3, 5), (16, 5), (7, 3)])
@pytest.mark.parametrize("pre", [0, 3])
def test_pair_gemm_protocol_random_schedules(tiles, nkt, stages, pre):
    for seed in range(6):
        run(tiles, nkt, stages, pre, seed)
