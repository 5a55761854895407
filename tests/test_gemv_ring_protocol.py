"""The shared-memory ring of the quantized GEMV (gemv_kernel, gb_gemv.cu),
modelled on the CPU: one producer issues stage k (K consecutive units) into
slot k mod NS once slot's previous stage was released (a parity wait on
empty[s]); each copy lands after a random delay, so copies of different slots
complete out of order; consumer warp w takes units w, w+W, w+2W, ... (stage
j >> log2 K), waits on full[s] with the phase parity (k / NS) & 1, reads the
slot and arrives on empty[s] (count K).

An mbarrier parity wait only tells the current phase's parity, so a waiter
two phases behind cannot be told from one that is on time. A warp takes every
dk = W/K-th stage; when dk does not divide NS, the stage that last used its
next slot (k - NS) belonged to other warps and may still be in flight, and a
parity wait for k alone would accept the completed phase before it. The kernel
therefore first waits for the release of stage k - NS (empty[s], parity
ph ^ 1). This model checks, for every ring shape the launcher can choose
(W = 8 or 16 consumer warps, K a power of two <= W, dk <= NS <= 8), that with
that wait every read sees its own stage and nothing deadlocks, and that
without it every shape whose stride dk does not divide NS reads early (the
check has the power to see the race)."""
import random

import pytest

MAX_STAGES = 8


def shapes():
    for W in (8, 16):
        K = 1
        while K <= W:
            dk = W // K
            for ns in range(max(2, dk), MAX_STAGES + 1):
                yield W, K, ns
            K *= 2


def simulate(W, K, NS, units, seed, prewait=True):
    """Random interleaving of the producer, the W consumer warps and the copy
    landings. Returns (early_reads, deadlocked)."""
    rng = random.Random(seed)
    nst = (units + K - 1) // K
    dk = W // K
    use_pre = prewait and NS % dk != 0
    full_n = [0] * NS      # completed phases of full[s]
    empty_n = [0] * NS     # completed phases of empty[s]
    empty_arr = [0] * NS   # arrivals in empty[s]'s current phase
    slot = [None] * NS     # stage whose bytes are in the slot
    inflight = []          # (slot, stage) copies not landed yet
    pk = 0                 # producer: next stage to issue
    warp_j = list(range(W))
    warp_pre = [False] * W  # the pre-wait of the warp's current unit is done
    early = 0

    def done(parity, n):  # mbarrier.try_wait.parity
        return (n & 1) != parity

    while True:
        actors = []
        if pk < nst:
            s = pk % NS
            if pk < NS or done(((pk // NS) - 1) & 1, empty_n[s]):
                actors.append(("p",))
        for w in range(W):
            j = warp_j[w]
            if j >= units:
                continue
            k = j // K
            s, ph = k % NS, (k // NS) & 1
            if use_pre and k >= NS and not warp_pre[w]:
                if done(ph ^ 1, empty_n[s]):
                    actors.append(("pre", w))
            elif done(ph, full_n[s]):
                actors.append(("c", w))
        # landings are chosen less often than the other actors, so copies stay
        # in flight while the warps run ahead
        for c in inflight:
            if rng.random() < 0.35:
                actors.append(("l", c))
        if not actors:
            if inflight:
                continue  # only landings left: draw again
            return early, any(warp_j[w] < units for w in range(W))
        a = rng.choice(actors)
        if a[0] == "p":
            s = pk % NS
            inflight.append((s, pk))
            pk += 1
        elif a[0] == "l":
            s, k = a[1]
            inflight.remove(a[1])
            slot[s] = k
            full_n[s] += 1
        elif a[0] == "pre":
            warp_pre[a[1]] = True
        else:
            w = a[1]
            j = warp_j[w]
            k = j // K
            s = k % NS
            if slot[s] != k:
                early += 1
            empty_arr[s] += 1
            if empty_arr[s] == K:
                empty_arr[s] = 0
                empty_n[s] += 1
            warp_j[w] = j + W
            warp_pre[w] = False


UNITS = (16, 56, 97)


@pytest.mark.parametrize("W,K,NS", list(shapes()))
def test_ring_reads_its_own_stage(W, K, NS):
    for units in UNITS:
        for seed in range(3):
            early, dead = simulate(W, K, NS, units, seed)
            assert not dead, f"deadlock W={W} K={K} NS={NS} units={units} seed={seed}"
            assert early == 0, f"{early} early reads W={W} K={K} NS={NS} units={units} seed={seed}"


def test_without_the_prewait_every_such_shape_reads_early():
    need = [(W, K, NS) for W, K, NS in shapes() if NS % (W // K) != 0]
    bad = [sh for sh in need if any(simulate(*sh, 97, seed, prewait=False)[0] for seed in range(6))]
    assert need and bad == need, f"the model missed the race for {sorted(set(need) - set(bad))}"
