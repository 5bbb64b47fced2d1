"""Model check of the chunked kernel's pair-release protocol (CPU only).

The tcgen05 kernel hands chunk pairs from two MMA warps to the epilogue warps
and back (f16acc_b200/csrc/tc_gemm.cuh, MMA-issuer and epilogue branches;
f16acc_b200/csrc/tc_epilogue.cuh, PairRing):

* hand-off n goes through pair b = n & 1 and is issued by MMA warp b, which
  commits it to tfull[b];
* every epilogue warp consumes the hand-offs in order and releases each with
  one `bar.arrive` on named barrier b;
* before issuing into pair b again, MMA warp b `bar.sync`s on that barrier (a
  round = the MMA warp + every epilogue warp), checking the abort flag before
  the `bar.sync` only (it issues right after the round completes, even when an
  abort completed it, and stops at its next check); at a normal end it
  reclaims its last hand-off;
* an epilogue warp that leaves early raises the abort flag and arrives once
  for the next hand-off of each pair if that hand-off was issued (its tfull
  completes within a bound).

`bar.sync` cannot time out, so the kernel relies on this protocol never
leaving an MMA warp in a round that cannot fill, and never putting two
arrivals of one warp into one round (hardware barriers only count).  This
test runs the protocol under random interleavings, random issue delays and
injected timeouts, with a model of the hardware barrier (a counter that
releases its waiters and resets when it reaches the thread count), and checks
both properties.  It checks the design, not the CUDA code; the kernel's
normal path is covered by the GPU parity tests.
"""

import random

import pytest


class Barrier:
    """Hardware named barrier: arrivals counted per warp; the round completes
    when the count reaches `need`, releasing the waiters."""

    def __init__(self, need):
        self.need = need
        self.count = 0
        self.round = 0
        self.contrib = set()  # warps that arrived in the current round
        self.waiters = set()
        self.overfill = False

    def _add(self, who):
        if who in self.contrib:
            self.overfill = True
        self.contrib.add(who)
        self.count += 1
        if self.count == self.need:
            self.count = 0
            self.round += 1
            self.contrib = set()
            released, self.waiters = self.waiters, set()
            return released
        return set()

    def arrive(self, who):
        self._add(who)

    def sync(self, who):
        """Returns the round the caller waits for completion of."""
        r = self.round
        self.waiters.add(who)
        self._add(who)
        return r


def run_protocol(seed, n_pairs, n_epi, fail_epi_at=None, fail_mma_at=None, third_party_abort_at=None,
                 naive_exit=False, wait_limit=3000):
    rng = random.Random(seed)
    bars = [Barrier(1 + n_epi), Barrier(1 + n_epi)]
    state = {"abort": False, "issued": set(), "step": 0}

    def mma(w):
        pending = False
        normal_end = False
        n = w
        done = False
        while n < n_pairs:
            # wait for the smem stage (bounded): may give up when aborting
            while rng.random() < 0.3:
                yield "spin"
            if fail_mma_at is not None and (w, n) == fail_mma_at:
                state["abort"] = True
                done = True
                break
            if state["abort"]:
                done = True
                break
            if pending:
                r = bars[w].sync(("mma", w))
                while bars[w].round == r:
                    yield "blocked"
                pending = False
            state["issued"].add(n)
            pending = True
            n += 2
        if not done:
            normal_end = True
        if normal_end and pending and not state["abort"]:
            r = bars[w].sync(("mma", w))
            while bars[w].round == r:
                yield "blocked"

    def epilogue(e):
        n = 0
        finished = True
        while n < n_pairs:
            # bounded wait for tfull(n): gives up on the abort flag or an injected timeout
            waited = 0
            while n not in state["issued"]:
                waited += 1
                if fail_epi_at is not None and (e, n) == fail_epi_at and waited > 3:
                    state["abort"] = True
                    break
                if waited > wait_limit:  # the kernel's time limit on the wait
                    state["abort"] = True
                    break
                if state["abort"] and rng.random() < 0.5:
                    break
                yield "spin"
            if n not in state["issued"]:
                finished = False
                break
            while rng.random() < 0.3:  # TMEM loads
                yield "spin"
            bars[n & 1].arrive(("epi", e))
            while rng.random() < 0.5:  # adds
                yield "spin"
            n += 1
        if not finished:
            state["abort"] = True
            if naive_exit:  # planted mistake: arrive on both barriers whatever was issued
                bars[0].arrive(("epi", e))
                bars[1].arrive(("epi", e))
                return
            # release the next hand-off of each pair if it was issued (bounded wait for its tfull)
            for nn in (n, n + 1):
                if nn >= n_pairs:
                    continue
                for _ in range(rng.randint(0, 20)):
                    if nn in state["issued"]:
                        break
                    yield "spin"
                if nn in state["issued"]:
                    bars[nn & 1].arrive(("epi", e))

    agents = {("mma", 0): mma(0), ("mma", 1): mma(1)}
    for e in range(n_epi):
        agents[("epi", e)] = epilogue(e)
    last = {k: "spin" for k in agents}
    steps = 0
    while agents:
        steps += 1
        if third_party_abort_at is not None and steps == third_party_abort_at:
            state["abort"] = True
        if steps > 200000:
            return "livelock", bars
        runnable = [k for k in agents if last[k] != "blocked" or k[0] != "mma" or not _blocked(bars, k)]
        if not runnable:
            return "deadlock", bars
        k = rng.choice(runnable)
        try:
            last[k] = next(agents[k])
        except StopIteration:
            del agents[k]
    return "ok", bars


def _blocked(bars, k):
    return k in bars[k[1]].waiters


@pytest.mark.parametrize("seed", range(40))
def test_normal_runs_fill_every_round_exactly(seed):
    rng = random.Random(1000 + seed)
    n_pairs = rng.randint(1, 13)
    n_epi = rng.choice([1, 2, 4, 8])
    result, bars = run_protocol(seed, n_pairs, n_epi)
    assert result == "ok"
    assert not any(b.overfill for b in bars)
    # every hand-off into a pair is one completed round, nothing left half full
    for b, bar in enumerate(bars):
        assert bar.round == len(range(b, n_pairs, 2))
        assert bar.count == 0


@pytest.mark.parametrize("seed", range(150))
def test_aborts_never_hang_or_overfill(seed):
    rng = random.Random(seed)
    n_pairs = rng.randint(2, 12)
    n_epi = rng.choice([1, 2, 4, 8])
    kind = seed % 3
    kw = {}
    if kind == 0:
        kw["fail_epi_at"] = (rng.randrange(n_epi), rng.randrange(n_pairs))
    elif kind == 1:
        kw["fail_mma_at"] = (rng.randrange(2), rng.randrange(n_pairs))
    else:
        kw["third_party_abort_at"] = rng.randint(1, 400)
    result, bars = run_protocol(seed, n_pairs, n_epi, **kw)
    assert result == "ok", (result, kw)
    assert not any(b.overfill for b in bars), kw


def test_model_detects_a_broken_exit_rule():
    """Planted mistake: epilogue warps that leave early arrive on both barriers
    unconditionally.  Some interleaving must then overfill a round (or strand an
    MMA warp), which shows the checks above have teeth."""
    bad = 0
    for seed in range(300):
        rng = random.Random(seed)
        n_pairs = rng.randint(4, 12)
        n_epi = rng.choice([2, 4])
        fail = (rng.randrange(n_epi), rng.randrange(1, n_pairs))
        result, bars = run_protocol(seed, n_pairs, n_epi, fail_epi_at=fail, naive_exit=True)
        if result != "ok" or any(b.overfill for b in bars):
            bad += 1
    assert bad > 0
