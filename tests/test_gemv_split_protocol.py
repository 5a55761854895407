"""The cross-CTA combine of row-blocks that a GEMV launch splits between CTAs
(gemv_kernel, gb_gemv.cu), modelled on the CPU with random interleavings.

CTA b of G owns units [U*b/G, U*(b+1)/G) (ubeg); a row-block is upr
consecutive units. A CTA whose range covers only part of a row-block stores
its partial in its slot (b, which): which = 0 when the row-block is its first
segment, 1 when it is its last. It then makes the store visible (fence) and adds
its unit count to the row-block's counter. The CTA whose addition completes
the count (upr) reads the slots of every CTA that touches the row-block, in
CTA order, resets the counter and runs the epilogue.

Checked over many launches of each shape, every one a fresh random
interleaving of the CTAs' steps:
- exactly one CTA finishes each split row-block, and only after every
  partial is in its slot;
- the finished value is the same bits whatever the order of arrival: the
  partials summed in CTA order;
- every counter is zero when the launch ends, so the next replay of a CUDA
  graph starts clean without a memset;
- cta_of_unit (the CTA owning a unit) agrees with the ranges.

This covers the shapes of the 8B (gate/up 14,336 units, lm_head 64,128), of the
70B's wider matrices, and some small ragged ones."""
import random

import numpy as np
import pytest


def ubeg(U, G, b):
    return (U * b) // G


def cta_of_unit(U, G, u):
    b = (u * G) // U
    while b > 0 and ubeg(U, G, b) > u:
        b -= 1
    while b + 1 < G and ubeg(U, G, b + 1) <= u:
        b += 1
    return b


def launch(U, G, upr, partial, counter, rng):
    """One launch. partial(b, rb) is CTA b's float32 partial of row-block rb.
    Returns {rb: value} of the finished split row-blocks."""
    slots = {}
    # each CTA's split segments, as a list of steps: (store, add-and-maybe-finish)
    work = []
    for b in range(G):
        c0, c1 = ubeg(U, G, b), ubeg(U, G, b + 1)
        if c0 == c1:
            continue
        rb = c0 // upr
        while rb * upr < c1:
            R0, R1 = rb * upr, rb * upr + upr
            t0, t1 = max(c0, R0), min(c1, R1)
            if not (t0 == R0 and t1 == R1):
                which = 0 if c0 >= R0 else 1
                work.append([b, rb, which, t1 - t0, 0])  # last field: next step
            rb += 1
    finished = {}
    pending = list(range(len(work)))
    while pending:
        i = rng.choice(pending)
        b, rb, which, n, step = work[i]
        if step == 0:  # store the partial, then the fence
            slots[(b, which)] = partial(b, rb)
            work[i][4] = 1
            continue
        pending.remove(i)
        counter[rb] += n  # atomicAdd
        if counter[rb] == upr:
            assert rb not in finished, "two CTAs finished one row-block"
            R0, R1 = rb * upr, rb * upr + upr
            bf, bl = cta_of_unit(U, G, R0), cta_of_unit(U, G, R1 - 1)
            z = np.float32(0)
            for b2 in range(bf, bl + 1):
                c0, c1 = ubeg(U, G, b2), ubeg(U, G, b2 + 1)
                if c0 == c1:
                    continue
                key = (b2, 0 if c0 >= R0 else 1)
                assert key in slots, "a partial read before it was stored"
                z = np.float32(z + slots[key])
            counter[rb] = 0
            finished[rb] = z
    return finished


SHAPES = [  # (units, CTAs, units per row-block)
    (14336, 148, 32),   # 8B gate/up pairs
    (64128, 148, 16),   # lm_head, 128256 rows
    (7168, 148, 56),    # a down projection on a persistent grid
    (28672, 148, 64),   # 70B down, 28672 columns
    (984, 37, 24),
    (91, 13, 7),
    (48, 33, 16),       # fewer units per CTA than a row-block: up to 12 CTAs share one
]  # a launch's units are always whole row-blocks (units = row-blocks x upr)


@pytest.mark.parametrize("U,G,upr", SHAPES)
def test_split_rowblocks_finish_once_in_cta_order(U, G, upr):
    for u in range(0, U, max(1, U // 997)):
        b = cta_of_unit(U, G, u)
        assert ubeg(U, G, b) <= u < ubeg(U, G, b + 1)
    assert U % upr == 0
    nrb = U // upr
    vals = np.random.default_rng(U + G).standard_normal((G, nrb)).astype(np.float32)
    partial = lambda b, rb: vals[b, rb]  # noqa: E731
    counter = [0] * nrb
    first = None
    for launch_no in range(6):
        got = launch(U, G, upr, partial, counter, random.Random(1000 * launch_no + G))
        assert all(c == 0 for c in counter), "a counter left non-zero for the next replay"
        if first is None:
            first = got
            # the split row-blocks are exactly those no single CTA covers
            for rb in range(U // upr):
                owners = {cta_of_unit(U, G, rb * upr), cta_of_unit(U, G, rb * upr + upr - 1)}
                assert (rb in got) == (len(owners) > 1)
        else:
            assert got.keys() == first.keys()
            for rb in got:
                assert got[rb].tobytes() == first[rb].tobytes(), "the sum depends on arrival order"
