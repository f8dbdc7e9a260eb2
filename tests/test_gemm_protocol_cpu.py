"""A CPU model of the persistent NVFP4 GEMM's barrier protocol (gemm_persistent_kernel in
csrc/nvfp4_gemm.cu), run under random schedules.

One CTA walks tiles t = cta, cta + grid, ...; its producer fills a ring of `stages` slots
(full[s]: TMA bytes; empty[s]: the MMA's commit after consuming the slot), the MMA lane
accumulates each tile into TMEM accumulator lt % 2 (accf[b]: commit when the tile is done;
acce[b]: the epilogue has drained it).  For the grouped (MoE) form the routing leaves a prefix
of the operand tiles in use and every role stops at the first tile whose expert is < 0.
Checks: every run ends (no deadlock), all three roles process the same tiles, no parity wait is
more than one phase behind, no ring slot is refilled before the MMA consumed it and no
accumulator is overwritten before the epilogue drained it."""
import random

import pytest


class Bar:
    def __init__(self, count=1):
        self.count, self.pending, self.done = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.done += 1
            self.pending = self.count


def run(tiles, used, nkt, stages, seed):
    """tiles: the CTA's tile count; used: how many of them the routing filled (grouped) ."""
    rnd = random.Random(seed)
    full = [Bar() for _ in range(stages)]
    empty = [Bar() for _ in range(stages)]
    accf, acce = [Bar(), Bar()], [Bar(), Bar()]
    slot_use = {}      # slot -> (use index, consumed?)
    acc_state = {}     # accumulator -> (tile, drained?)
    seen = {"p": [], "m": [], "e": []}
    async_q, tick = [], [0]

    def expert_ok(i):
        return i < used

    def after(fn):
        ready = tick[0] + rnd.randint(1, 5)
        if async_q:
            ready = max(ready, async_q[-1][0])
        async_q.append((ready, fn))

    def wait(b, parity_index):
        while b.done <= parity_index:
            yield
        assert b.done <= parity_index + 2, "parity alias"

    def producer():
        it = 0
        for i in range(tiles):
            if not expert_ok(i):
                break
            seen["p"].append(i)
            for _ in range(nkt):
                s = it % stages
                if it >= stages:
                    yield from wait(empty[s], it // stages - 1)
                assert slot_use.get(s, (None, True))[1], "ring slot refilled before the MMA consumed it"
                slot_use[s] = (it, False)
                after(lambda s=s: full[s].arrive())
                it += 1

    def mma():
        it = 0
        for lt in range(tiles):
            if not expert_ok(lt):
                break
            seen["m"].append(lt)
            b, use = lt & 1, lt >> 1
            if use > 0:
                yield from wait(acce[b], use - 1)
            assert acc_state.get(b, (None, True))[1], "accumulator overwritten before the epilogue drained it"
            acc_state[b] = (lt, False)
            for _ in range(nkt):
                s = it % stages
                yield from wait(full[s], it // stages)
                assert slot_use[s][0] == it

                def consumed(s=s):
                    slot_use[s] = (slot_use[s][0], True)
                    empty[s].arrive()
                after(consumed)
                it += 1
            after(lambda b=b: accf[b].arrive())

    def epilogue():
        for lt in range(tiles):
            if not expert_ok(lt):
                break
            seen["e"].append(lt)
            b, use = lt & 1, lt >> 1
            yield from wait(accf[b], use)
            assert acc_state[b][0] == lt
            yield
            acc_state[b] = (lt, True)
            acce[b].arrive()

    live = [producer(), mma(), epilogue()]
    for _ in range(100000):
        tick[0] += 1
        while async_q and async_q[0][0] <= tick[0]:
            async_q.pop(0)[1]()
        if not live and not async_q:
            assert seen["p"] == seen["m"] == seen["e"] == list(range(min(used, tiles)))
            return
        rnd.shuffle(live)
        for r in list(live)[: rnd.randint(1, len(live))]:
            try:
                next(r)
            except StopIteration:
                live.remove(r)
    raise AssertionError("the protocol did not finish (deadlock)")


@pytest.mark.parametrize("tiles,used", [(1, 1), (3, 3), (7, 7), (7, 4), (7, 0), (9, 1)])
@pytest.mark.parametrize("nkt,stages", [(1, 2), (8, 6), (16, 4), (3, 8)])
def test_persistent_gemm_protocol_random_schedules(tiles, used, nkt, stages):
    for seed in range(25):
        run(tiles, used, nkt, stages, seed)
