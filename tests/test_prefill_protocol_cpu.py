"""A CPU model of the prefill attention kernel's barrier protocol (csrc/prefill_attention.cu,
tcgen05 form), run under many random schedules.

Each role of the kernel (producer, converter warps, MMA issuer, softmax warps of each query
tile) is a generator that performs the kernel's waits and arrivals in the kernel's order, with
the kernel's slot / phase arithmetic.  Asynchronous work (TMA completion, tcgen05.commit
arrivals) completes later, in issue order, after random delays.  The model checks that
  * every run finishes (no deadlock), for block counts around the ring sizes;
  * no parity wait is ambiguous: when a role waits for phase k of a barrier, the barrier has
    completed at most k + 1 phases (a barrier two phases ahead would alias the parity);
  * no buffer is overwritten while a reader may still use it (staging slots, K/V operand slots,
    S buffers, the single P tile per query tile)."""
import random

import pytest

NSTG, NKV, NT, NCONV, NSOFT = 2, 3, 2, 4, 4  # the kernel's constants


class Bar:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.done = 0  # completed phases

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.done += 1
            self.pending = self.count


def run(nblk, seed):
    rnd = random.Random(seed)
    B = {}

    def bar(name, count=1):
        if name not in B:
            B[name] = Bar(count)
        return B[name]

    for s in range(NSTG):
        bar(("e_full", s), 1), bar(("e_empty", s), NCONV)
    for i in range(NKV):
        bar(("kv_full", i), NCONV), bar(("kv_empty", i), 1)
    for t in range(NT):
        for b in range(2):
            bar(("s_full", t, b), 1)
        bar(("p_full", t), NSOFT), bar(("o_done", t), 1)
    bar("q_ready", NCONV), bar("fin", 1)

    # buffer state for hazard checks
    staged = {}      # staging slot -> block held (written by TMA)
    kv_slot = {}     # K/V operand slot -> block held
    kv_readers = {}  # K/V slot -> set of (kind, tile) still to read it
    s_buf = {}       # (t, b) -> block held, consumed flag
    p_tile = {}      # t -> block written, read by P.V?
    async_q = []     # tensor-pipe / TMA completions, in issue order: (ready_tick, fn)
    tick = [0]

    def wait(name, k):
        b = B[name]
        while b.done <= k:
            yield
        assert b.done <= k + 2, f"{name}: waiting for phase {k}, {b.done} completed (parity alias)"

    def after(fn, delay=None):
        ready = tick[0] + (delay if delay is not None else rnd.randint(1, 6))
        if async_q:
            ready = max(ready, async_q[-1][0])  # in order
        async_q.append((ready, fn))

    def producer():
        for j in range(nblk):
            s = j % NSTG
            if j >= NSTG:
                yield from wait(("e_empty", s), j // NSTG - 1)
            assert staged.get(s, (None, True))[1], "staging slot refilled before the converters released it"
            staged[s] = (j, False)
            after(lambda s=s: B[("e_full", s)].arrive())

    def converter(w):
        B["q_ready"].arrive()
        for j in range(nblk):
            s, kb = j % NSTG, j % NKV
            yield from wait(("e_full", s), j // NSTG)
            assert staged[s][0] == j
            if j >= NKV:
                yield from wait(("kv_empty", kb), j // NKV - 1)
            if w == 0:
                assert not kv_readers.get(kb), "K/V slot rewritten while the MMAs still read it"
                kv_slot[kb] = j
                kv_readers[kb] = {("pv", t) for t in range(NT)} | {("s", t) for t in range(NT)}
            yield
            B[("kv_full", kb)].arrive()
            B[("e_empty", s)].arrive()
            if B[("e_empty", s)].pending == NCONV:  # all converter warps released it
                staged[s] = (j, True)

    def mma():
        if nblk == 0:
            return
        yield from wait("q_ready", 0)
        yield from wait(("kv_full", 0), 0)

        def issue_s(j):
            kb = j % NKV
            assert kv_slot.get(kb) == j
            for t in range(NT):
                key = (t, j & 1)
                prev = s_buf.get(key)
                assert prev is None or prev[1], "S buffer overwritten before its softmax read it"
                s_buf[key] = (j, False)
                kv_readers[kb].discard(("s", t))
                after(lambda t=t, j=j: B[("s_full", t, j & 1)].arrive())

        issue_s(0)
        for j in range(nblk):
            if j + 1 < nblk:
                yield from wait(("kv_full", (j + 1) % NKV), (j + 1) // NKV)
                issue_s(j + 1)
            for t in range(NT):
                yield from wait(("p_full", t), j)
                assert p_tile[t] == (j, False)

                def pv_done(t=t, j=j):
                    p_tile[t] = (j, True)
                    kv_readers[j % NKV].discard(("pv", t))
                    B[("o_done", t)].arrive()
                after(pv_done)
            after(lambda j=j: B[("kv_empty", j % NKV)].arrive())
        after(lambda: B["fin"].arrive())
        yield from wait("fin", 0)

    def softmax(t, w):
        for j in range(nblk):
            sb = j & 1
            yield from wait(("s_full", t, sb), j >> 1)
            assert s_buf[(t, sb)][0] == j
            kv = B[("kv_full", j % NKV)]
            assert kv.done > j // NKV, "page flags read before their slot was filled"
            yield
            if j > 0:
                yield from wait(("o_done", t), j - 1)
            if w == 0:
                prev = p_tile.get(t)
                assert prev is None or prev[1], "P tile rewritten before its P.V completed"
                p_tile[t] = (j, False)
            B[("p_full", t)].arrive()
            if B[("p_full", t)].pending == NSOFT:  # the warpgroup has consumed S_j
                s_buf[(t, sb)] = (j, True)
        if nblk:
            yield from wait(("o_done", t), nblk - 1)

    roles = [producer(), mma()] + [converter(w) for w in range(NCONV)]
    roles += [softmax(t, w) for t in range(NT) for w in range(NSOFT)]
    live = list(roles)
    for _ in range(200000):
        tick[0] += 1
        while async_q and async_q[0][0] <= tick[0]:
            async_q.pop(0)[1]()
        if not live and not async_q:
            return
        rnd.shuffle(live)
        for r in list(live)[: rnd.randint(1, len(live) or 1)]:
            try:
                next(r)
            except StopIteration:
                live.remove(r)
    raise AssertionError("the protocol did not finish (deadlock)")


@pytest.mark.parametrize("nblk", [0, 1, 2, 3, 4, 5, 7, 12])
def test_prefill_barrier_protocol_random_schedules(nblk):
    for seed in range(40):
        run(nblk, seed)
