"""A CPU model of the tensor-parallel peer-memory reduction protocol of the decode engine
(GEMM epilogues writing tagged 8-byte words into every rank's inbox, csrc/nvfp4_gemm.cu;
the RMSNorm on each rank polling its inbox, csrc/parts.cuh load_parts_tagged), run under
random interleavings of W ranks with no barrier between them.

Per step e and layer l every rank runs, in stream order: the o_proj GEMM (writes its word into
the o-inbox of every rank, tag (e, l, o)), the RMSNorm that waits for all ranks' o-words in its
own o-inbox, the down GEMM (writes the down-inbox of every rank, tag (e, l, down)), and the
RMSNorm that waits for all down-words.  A GEMM's writes to the different ranks land in any
order.  Tags are epoch * 2L + 2 l + kind + 1, as the engine sets them.
Checks: every run ends (no rank waits for a tag that was already overwritten), and no word is
overwritten before the rank that owns the inbox has consumed it: the reuse rule (a rank rewrites
a peer's o-inbox only after consuming that peer's down-words of the previous layer, which the
peer wrote after reading its own o-inbox) needs no barrier."""
import random

import pytest


def run(world, layers, steps, seed):
    rnd = random.Random(seed)
    tag_mul = 2 * layers
    # inbox[dst][kind][src] = (tag, consumed)
    inbox = [[[(0, True) for _ in range(world)] for _ in range(2)] for _ in range(world)]

    def tag(e, l, kind):
        return e * tag_mul + 2 * l + kind + 1

    def gemm(r, e, l, kind):
        dsts = list(range(world))
        rnd.shuffle(dsts)
        for p in dsts:  # the epilogue's words reach the ranks in any order
            old_tag, consumed = inbox[p][kind][r]
            assert consumed, f"rank {r} overwrote rank {p}'s {('o', 'down')[kind]} word (tag {old_tag}) before it was read"
            inbox[p][kind][r] = (tag(e, l, kind), False)
            yield

    def rmsnorm(r, e, l, kind):
        want = tag(e, l, kind)
        for q in range(world):
            while inbox[r][kind][q][0] != want:
                assert inbox[r][kind][q][0] < want, "a newer tag replaced the awaited one"
                yield
        for q in range(world):
            inbox[r][kind][q] = (want, True)
        yield

    def rank(r):
        for e in range(steps):
            for l in range(layers):
                yield from gemm(r, e, l, 0)
                yield from rmsnorm(r, e, l, 0)
                yield from gemm(r, e, l, 1)
                yield from rmsnorm(r, e, l, 1)

    live = [rank(r) for r in range(world)]
    for _ in range(200000):
        if not live:
            return
        r = rnd.choice(live)
        try:
            next(r)
        except StopIteration:
            live.remove(r)
    raise AssertionError("a rank never saw its awaited tag (deadlock)")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_inbox_reuse_needs_no_barrier(world):
    for seed in range(30):
        run(world, layers=3, steps=3, seed=seed)


def test_single_inbox_for_both_kinds_would_be_unsafe():
    """Counter-check of the model: with one inbox shared by o and down words (kind forced to
    0 for the slots), a fast rank overwrites words its peers have not read yet."""
    def run_shared(seed):
        rnd = random.Random(seed)
        world, layers, steps = 4, 3, 2
        box = [[(0, True) for _ in range(world)] for _ in range(world)]
        tagn = [0]

        def rank(r):
            n = 0
            for _ in range(steps * layers * 2):
                n += 1
                dsts = list(range(world))
                rnd.shuffle(dsts)
                for p in dsts:
                    if not box[p][r][1]:
                        raise AssertionError("overwrite")
                    box[p][r] = (n, False)
                    yield
                for q in range(world):
                    while box[r][q][0] < n:
                        yield
                    if box[r][q][0] > n:
                        raise AssertionError("overwrite")
                for q in range(world):
                    box[r][q] = (n, True)
                yield
        live = [rank(r) for r in range(world)]
        for _ in range(100000):
            if not live:
                return False
            r = rnd.choice(live)
            try:
                next(r)
            except StopIteration:
                live.remove(r)
            except AssertionError:
                return True
        return True
    assert any(run_shared(s) for s in range(50))
