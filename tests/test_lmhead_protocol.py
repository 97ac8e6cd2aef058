"""CPU model of the LM head's mbarrier protocol (lmhead_tc_kernel in
csrc/g4s_lmhead.cu): the weight-copy warp, the activation-copy warp, the two
MMA warps and the eight dequantizing warps, with bulk copies completing in any
order and each MMA warp's commits completing in issue order, interleaved at
random.  A barrier wait there is a parity test (mbarrier.try_wait.parity): it
succeeds when the barrier's current phase has the other parity, so it cannot
tell the phase it wants from one two phases behind.  The model checks, for the
ring depths the kernel builds with and a few others, that every wait that
succeeds finds its phase complete and no later one (the parity argument in the
kernel's comments), and that the pipeline always finishes."""
import random

import pytest


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.done = count, count, 0   # done = completed phases

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def ready(self, need):
        """Parity wait for the need-th completion (parity (need - 1) & 1)."""
        ok = (self.done & 1) != ((need - 1) & 1)
        if ok:
            assert self.done >= need, "a parity wait passed an earlier phase"
            assert self.done <= need, "a barrier ran a whole phase past its waiter"
        return ok


def run(nch, RS, BS, AS, seed):
    rng = random.Random(seed)
    raw_full = [Bar(1) for _ in range(RS)]
    raw_empty = [Bar(8) for _ in range(RS)]
    b_full = [Bar(1) for _ in range(BS)]
    b_empty = [Bar(2) for _ in range(BS)]
    a_full = [[Bar(5) for _ in range(AS)] for _ in range(2)]
    ab_empty = [[Bar(1) for _ in range(AS)] for _ in range(2)]
    asyncs = []            # pending completions: (kind, fn), copies in any order
    commits = [[], []]     # per MMA warp: committed barriers in issue order

    def raw_loader():
        for c in range(nch):
            while not raw_empty[c % RS].ready(c // RS):
                yield
            asyncs.append(raw_full[c % RS].arrive)

    def b_loader():
        lead = BS - AS

        def issue(c):
            while not b_empty[c % BS].ready(c // BS):
                yield
            asyncs.append(b_full[c % BS].arrive)
        for c in range(min(lead, nch)):
            yield from issue(c)
        for c in range(nch):
            a = c % AS
            while not (b_full[c % BS].ready(c // BS + 1) and ab_empty[0][a].ready(c // AS)
                       and ab_empty[1][a].ready(c // AS)):
                yield
            a_full[0][a].arrive()
            a_full[1][a].arrive()
            if c + lead < nch:
                yield from issue(c + lead)

    def mma(mt):
        for c in range(nch):
            while not a_full[mt][c % AS].ready(c // AS + 1):
                yield
            commits[mt].append((ab_empty[mt][c % AS], b_empty[c % BS]))

    def dequant(w):
        mt = w // 4
        for c in range(nch):
            while not (raw_full[c % RS].ready(c // RS + 1) and ab_empty[mt][c % AS].ready(c // AS)):
                yield
            raw_empty[c % RS].arrive()
            a_full[mt][c % AS].arrive()

    roles = [raw_loader(), b_loader(), mma(0), mma(1)] + [dequant(w) for w in range(8)]
    live = list(roles)
    for _ in range(10 ** 6):
        if not live and not asyncs and not commits[0] and not commits[1]:
            return
        choice = rng.random()
        if asyncs and choice < 0.3:
            asyncs.pop(rng.randrange(len(asyncs)))()
        elif (commits[0] or commits[1]) and choice < 0.5:
            mt = rng.choice([m for m in (0, 1) if commits[m]])
            for bar in commits[mt].pop(0):   # a commit completes after the MMAs before it
                bar.arrive()
        elif live:
            r = rng.choice(live)
            try:
                next(r)
            except StopIteration:
                live.remove(r)
    raise AssertionError("the pipeline did not finish (deadlock)")


@pytest.mark.parametrize("RS,BS,AS", [(6, 6, 2), (4, 8, 2), (8, 4, 2), (3, 3, 2), (8, 8, 6)])
def test_lmhead_barrier_protocol(RS, BS, AS):
    for seed in range(40):
        run(nch=40, RS=RS, BS=BS, AS=AS, seed=seed)
