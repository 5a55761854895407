"""The tensor-parallel exchange protocol of the decode step, modelled on the CPU
with real concurrency (no GPU): each rank is a process that owns a shared
buffer of 64-bit words [slots][dim] and, per step, writes its partial of every
exchange slot as (step + 1) << 32 | float bits in a random order with random
pauses (the row-split GEMV's CTAs finish in any order), then reads every rank's
word of each element, polling only while the tag is an older step (bounded),
and adds the values in rank order (peer_resid_tagged_kernel). A barrier per
step stands in for the argmax exchange that ends each decode step, which is
what keeps a rank from overwriting a slot before the others have read it.

Checked: no rank ever sums a word of another step, every rank obtains the
same bits, and those bits equal the rank-order float32 sum of the partials.
The step counter only grows, so a stale word can never carry the current tag."""
import multiprocessing as mp
import time

import numpy as np
import pytest

SLOTS, DIM, STEPS = 3, 96, 6
POLL_LIMIT = 2_000_000


def partial(step, slot, rank):
    rng = np.random.default_rng([step, slot, rank])
    return rng.standard_normal(DIM).astype(np.float32)


def expected(step, slot, world):
    acc = np.zeros(DIM, dtype=np.float32)
    for q in range(world):
        acc = (acc + partial(step, slot, q)).astype(np.float32)
    return acc


def _rank(rank, world, names, barrier, out_q):
    from multiprocessing import shared_memory

    shms = [shared_memory.SharedMemory(name=n) for n in names]
    try:
        bufs = [np.ndarray((SLOTS, DIM), dtype=np.uint64, buffer=s.buf) for s in shms]
        rng = np.random.default_rng(1000 + rank)
        results, stale_seen = [], 0
        for step in range(STEPS):
            tag = np.uint64(step + 1) << np.uint64(32)
            for slot in range(SLOTS):
                # this rank's words, row-blocks in a random order with pauses
                bits = partial(step, slot, rank).view(np.uint32).astype(np.uint64)
                for blk in rng.permutation(DIM // 32):
                    lo, hi = blk * 32, blk * 32 + 32
                    bufs[rank][slot, lo:hi] = bits[lo:hi] | tag
                    if rng.random() < 0.3:
                        time.sleep(rng.random() * 1e-3)
                # the exchange: every rank's word of each element, polled while stale
                acc = np.zeros(DIM, dtype=np.float32)
                for q in range(world):
                    w = bufs[q][slot].copy()
                    polls = 0
                    while True:
                        fresh = (w >> np.uint64(32)) == np.uint64(step + 1)
                        older = (w >> np.uint64(32)) < np.uint64(step + 1)
                        assert np.all(fresh | older), "a word from a later step"
                        if fresh.all():
                            break
                        stale_seen += int((~fresh).sum())
                        polls += 1
                        assert polls < POLL_LIMIT, "exchange wait ran out"
                        w[~fresh] = bufs[q][slot][~fresh]
                    vals = (w & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
                    acc = (acc + vals).astype(np.float32)
                results.append(acc.view(np.uint32).copy())
            barrier.wait(timeout=60)  # the step's argmax exchange
        out_q.put((rank, np.stack(results), stale_seen))
    finally:
        for s in shms:
            s.close()


@pytest.mark.parametrize("world", [2, 4])
def test_tagged_exchange_protocol(world):
    from multiprocessing import shared_memory

    ctx = mp.get_context("spawn")
    shms = [shared_memory.SharedMemory(create=True, size=SLOTS * DIM * 8) for _ in range(world)]
    try:
        for s in shms:
            np.ndarray((SLOTS, DIM), dtype=np.uint64, buffer=s.buf)[:] = 0
        barrier, out_q = ctx.Barrier(world), ctx.Queue()
        procs = [ctx.Process(target=_rank, args=(r, world, [s.name for s in shms], barrier, out_q))
                 for r in range(world)]
        for p in procs:
            p.start()
        got = dict()
        for _ in range(world):
            r, res, _stale = out_q.get(timeout=120)
            got[r] = res
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
        want = np.stack([expected(st, sl, world).view(np.uint32) for st in range(STEPS) for sl in range(SLOTS)])
        for r in range(world):
            assert np.array_equal(got[r], want), f"rank {r} summed other bits"
    finally:
        for s in shms:
            s.close()
            s.unlink()
