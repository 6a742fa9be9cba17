"""An executable model of the sharded prefill's peer-memory all-gather protocol
(fftsparse_b200/dist.py PeerGather, fftsparse_b200/csrc/peer.cu): every rank's
calls run in stream order

    attention(e)  stores its heads' rows into its own buffer slot e % 2 and into
                  the same slot of every peer (stores land at arbitrary times
                  while the kernel runs, all before it completes)
    signal(e)     stores e into its flag word in every rank's flag array
    wait(e)       until every flag word of its own array is >= e
    consume(e)    reads slot e % 2 (o_proj), before attention(e + 1)

while the ranks interleave arbitrarily.  Checks: what a rank consumes holds
epoch e from every rank, and no store of another epoch lands in a slot while it
is being consumed.  A planted mistake (a single buffer slot) must be caught.
"""
import random

import pytest


class Model:
    def __init__(self, world, calls, seed, slots=2):
        self.rng = random.Random(seed)
        self.W, self.E, self.slots = world, calls, slots
        # buf[r][slot][p] = epoch of rank p's rows in rank r's buffer slot
        self.buf = [[[0] * world for _ in range(slots)] for _ in range(world)]
        self.flags = [[0] * world for _ in range(world)]  # flags[r][p]: rank p's epoch, in r's array
        self.reading = [None] * world  # slot being consumed by rank r

    def rank(self, r):
        for e in range(1, self.E + 1):
            s = e % self.slots
            # attention(e): the rows for every destination land in some order
            dests = list(range(self.W))
            self.rng.shuffle(dests)
            for d in dests:
                assert self.reading[d] != s, f"rank {r} epoch {e} stored into slot {s} while rank {d} reads it"
                self.buf[d][s][r] = e
                yield
            # signal(e), after the kernel (stores visible system-wide first)
            for d in range(self.W):
                self.flags[d][r] = e
            yield
            # wait(e)
            while min(self.flags[r]) < e:
                yield
            # consume(e), spread over several steps
            self.reading[r] = s
            for _ in range(self.rng.randint(1, 3)):
                assert self.buf[r][s] == [e] * self.W, f"rank {r} consumed {self.buf[r][s]} at epoch {e}"
                yield
            self.reading[r] = None

    def run(self, max_steps=100000):
        roles = {r: self.rank(r) for r in range(self.W)}
        for _ in range(max_steps):
            if not roles:
                return
            r = self.rng.choice(list(roles))
            try:
                next(roles[r])
            except StopIteration:
                del roles[r]
        raise RuntimeError("deadlock")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_peer_gather_protocol(world):
    for seed in range(200):
        Model(world, 6, seed).run()


def test_model_catches_single_slot():
    with pytest.raises(AssertionError):
        for seed in range(500):
            Model(4, 6, seed, slots=1).run()
