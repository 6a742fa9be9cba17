"""An executable model of the attention kernel's barrier protocol
(fftsparse_b200/csrc/attn_fwd.cu): the TMA producer, the MMA issuer and the
softmax warps as coroutines; mbarriers with phase parity; TMA copies completing
in any order; tcgen05 operations completing in issue order.  Over random
interleavings, every wait must return after the event it is meant for (the S
tile, the P tile, the K / V stage contents, PV completion for a rescale of O),
no buffer may be overwritten while still needed, and every role must finish.
Planted protocol mistakes must be caught.  The model restates the kernel's
rings: K in 3 stages (released by the S MMA that read it), V in 2 (released by
the PV commit of the same S buffer), S/P double-buffered in TMEM, and the MMA
order S(0), S(1), then PV(n), S(n+2).
"""
import pytest

import random


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def ready(self, parity):
        return (self.phase & 1) != parity


class Sim:
    KS, VS = 3, 2

    def __init__(self, n, seed):
        self.rng = random.Random(seed)
        self.n = n
        self.BQ = Bar(1)
        self.BKF = [Bar(1) for _ in range(self.KS)]
        self.BKE = [Bar(1) for _ in range(self.KS)]
        self.BVF = [Bar(1) for _ in range(self.VS)]
        self.BSF = [Bar(1), Bar(1)]
        self.BPV = [Bar(1), Bar(1)]
        self.BPF = [Bar(128), Bar(128)]
        self.kst = [None] * self.KS
        self.vst = [None] * self.VS
        self.S = [None, None]   # per S buffer: ("S", n) or ("P", n)
        self.O = []
        self.mma_q, self.tma = [], []

    def step_tma(self):
        i = self.rng.randrange(len(self.tma))
        kind, st, tile, bar = self.tma.pop(i)
        (self.kst if kind == "K" else self.vst)[st] = tile
        bar.arrive()

    def step_mma(self):
        op = self.mma_q.pop(0)
        if op[0] == "S":
            _, n = op
            assert self.kst[n % self.KS] == n, f"S({n}) read K {self.kst[n % self.KS]}"
            b = n % 2
            if n >= 2:
                assert self.S[b] == ("P", n - 2) and (n - 2) in self.O, f"S({n}) overwrote {self.S[b]}"
            self.S[b] = ("S", n)
        elif op[0] == "PV":
            _, n = op
            assert self.S[n % 2] == ("P", n), f"PV({n}) read {self.S[n % 2]}"
            assert self.vst[n % self.VS] == n, f"PV({n}) read V {self.vst[n % self.VS]}"
            self.O.append(n)
        else:
            op[1].arrive()

    def producer(self):
        self.tma.append(("Q", 0, 0, self.BQ))

        def load(n, is_k):
            ns = self.KS if is_k else self.VS
            s = n % ns
            empty = (self.BKE if is_k else self.BPV)[s]
            while not empty.ready(((n // ns) & 1) ^ 1):
                yield
            self.tma.append(("K" if is_k else "V", s, n, (self.BKF if is_k else self.BVF)[s]))
        yield from load(0, True)
        for n in range(self.n):
            if n + 1 < self.n:
                yield from load(n + 1, True)
            yield from load(n, False)

    def mma(self):
        while not self.BQ.ready(0):
            yield

        def wait(bar, p):
            while not bar.ready(p):
                yield

        def issue_s(n):
            yield from wait(self.BKF[n % self.KS], (n // self.KS) & 1)
            self.mma_q += [("S", n), ("commit", self.BSF[n % 2]), ("commit", self.BKE[n % self.KS])]

        yield from issue_s(0)
        if self.n > 1:
            yield from issue_s(1)
        for n in range(self.n):
            s = n % 2
            yield from wait(self.BVF[s], (n >> 1) & 1)
            yield from wait(self.BPF[s], (n >> 1) & 1)
            self.mma_q += [("PV", n), ("commit", self.BPV[s])]
            if n + 2 < self.n:
                yield from issue_s(n + 2)

    def softmax(self):
        for n in range(self.n):
            sb = n % 2
            while not self.BSF[sb].ready((n >> 1) & 1):
                yield
            assert self.S[sb] == ("S", n), f"softmax {n} saw {self.S[sb]}"
            yield
            self.S[sb] = ("P", n)
            if n >= 1 and self.rng.random() < 0.3:  # rescale O: PV(n-1) must be complete
                while not self.BPV[(n - 1) % 2].ready(((n - 1) >> 1) & 1):
                    yield
                assert (n - 1) in self.O and n not in self.O
            self.BPF[sb].arrive(128)
        m = self.n - 1
        while not self.BPV[m % 2].ready((m >> 1) & 1):
            yield
        assert self.O == list(range(self.n)), self.O

    def run(self, max_steps=200000):
        roles = {"p": self.producer(), "m": self.mma(), "s": self.softmax()}
        done = set()
        for _ in range(max_steps):
            if len(done) == 3 and not self.mma_q and not self.tma:
                return
            ch = [r for r in roles if r not in done] + (["tma"] if self.tma else []) + (["tc"] if self.mma_q else [])
            c = self.rng.choice(ch)
            if c == "tma":
                self.step_tma()
            elif c == "tc":
                self.step_mma()
            else:
                try:
                    next(roles[c])
                except StopIteration:
                    done.add(c)
        raise RuntimeError(f"deadlock: done={done}")




@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8, 13])
def test_protocol_random_interleavings(n):
    for seed in range(60):
        Sim(n, seed).run()


def test_model_catches_a_missing_release_wait():
    class Early(Sim):  # producer reuses a V stage without waiting for the PV that reads it
        def producer(self):
            self.tma.append(("Q", 0, 0, self.BQ))

            def load(n, is_k):
                ns = self.KS if is_k else self.VS
                s = n % ns
                if is_k:
                    while not self.BKE[s].ready(((n // ns) & 1) ^ 1):
                        yield
                self.tma.append(("K" if is_k else "V", s, n, (self.BKF if is_k else self.BVF)[s]))
            yield from load(0, True)
            for n in range(self.n):
                if n + 1 < self.n:
                    yield from load(n + 1, True)
                yield from load(n, False)
    with pytest.raises((AssertionError, RuntimeError)):
        for seed in range(200):
            Early(5, seed).run(max_steps=20000)


def test_model_catches_s_issued_before_pv():
    class Eager(Sim):  # S(n+2) issued before PV(n): it would overwrite P(n) unread
        def mma(self):
            while not self.BQ.ready(0):
                yield

            def wait(bar, p):
                while not bar.ready(p):
                    yield

            def issue_s(n):
                yield from wait(self.BKF[n % self.KS], (n // self.KS) & 1)
                self.mma_q += [("S", n), ("commit", self.BSF[n % 2]), ("commit", self.BKE[n % self.KS])]
            yield from issue_s(0)
            if self.n > 1:
                yield from issue_s(1)
            for n in range(self.n):
                s = n % 2
                yield from wait(self.BVF[s], (n >> 1) & 1)
                yield from wait(self.BPF[s], (n >> 1) & 1)
                if n + 2 < self.n:
                    yield from issue_s(n + 2)
                self.mma_q += [("PV", n), ("commit", self.BPV[s])]
    with pytest.raises((AssertionError, RuntimeError)):
        for seed in range(200):
            Eager(5, seed).run(max_steps=20000)
