"""The sampling rule on the host (oracle/or_sample), no GPU: its exp against
float64, the seeded draw, greedy = model.Argmax, and the distributions it
draws from fixed logits against the closed-form probabilities (the
reference's roadmap proof for sampling: "distributions match a host
reference on fixed logits"). The device sampler is checked against this
rule token for token in test_sampler_gpu.py."""
import numpy as np
import pytest

import oracle_lib as orl


def softmax(z):
    z = np.asarray(z, np.float64)
    e = np.exp(z - z.max())
    return e / e.sum()


def draws(logits, n, **kw):
    return np.array([orl.sample(logits, counter=c, **kw) for c in range(n)])


def chi2_ok(counts, probs, n):
    # Pearson chi-square over the cells with expected count >= 5, p-value >= 1e-4
    from scipy.stats import chi2
    exp = probs * n
    keep = exp >= 5
    stat = (((counts - exp) ** 2) / np.where(exp > 0, exp, 1))[keep].sum()
    rest = exp[~keep].sum()
    if rest > 0:
        stat += (counts[~keep].sum() - rest) ** 2 / rest
    dof = keep.sum() - (0 if rest > 0 else 1)
    return chi2.sf(stat, dof) >= 1e-4, stat


def test_exp_nonpos_accuracy():
    xs = np.concatenate([-np.logspace(-8, np.log10(87), 20000), np.linspace(-87, 0, 20001)]).astype(np.float32)
    got = np.array([orl.exp_nonpos(float(x)) for x in xs], np.float64)
    want = np.exp(xs.astype(np.float64))
    ulp = np.spacing(want.astype(np.float32)).astype(np.float64)
    err = np.abs(got - want) / ulp
    assert err.max() <= 4.0, f"max error {err.max():.2f} ulp at x={xs[err.argmax()]}"
    assert orl.exp_nonpos(0.0) == 1.0
    assert orl.exp_nonpos(-88.0) == 0.0 and orl.exp_nonpos(float("-inf")) == 0.0
    assert orl.exp_nonpos(float("nan")) == 0.0


def test_uniform24():
    u = np.array([orl.uniform24(7, c) for c in range(20000)])
    assert u.min() >= 0.0 and u.max() < 1.0
    assert np.all((u * 2**24) == np.round(u * 2**24))  # 24-bit grid
    assert abs(u.mean() - 0.5) < 0.01 and len(np.unique(u)) > 19900
    assert orl.uniform24(7, 3) != orl.uniform24(8, 3)


def test_greedy_is_argmax():
    rng = np.random.default_rng(1)
    for n in (1, 5, 1000, 4097):
        x = rng.standard_normal(n).astype(np.float32)
        for t in (0.0, -1.0):
            assert orl.sample(x, temperature=t, counter=3) == orl.argmax(x)
        assert orl.sample(x, temperature=0.9, top_k=1, counter=3) == orl.argmax(x)
    x = np.array([1, 3, 3, 2], np.float32)  # ties: the first maximum
    assert orl.sample(x, temperature=0) == 1


def test_full_vocab_distribution():
    rng = np.random.default_rng(2)
    x = (2 * rng.standard_normal(40)).astype(np.float32)
    n = 20000
    for t in (0.7, 1.0, 1.6):
        got = np.bincount(draws(x, n, temperature=t, top_k=0, top_p=1.0, seed=5), minlength=40)
        ok, stat = chi2_ok(got, softmax(x.astype(np.float64) / t), n)
        assert ok, (t, stat)


def test_top_k_distribution():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(300).astype(np.float32)
    n, k = 20000, 8
    d = draws(x, n, temperature=1.0, top_k=k, top_p=1.0, seed=9)
    top = np.argsort(-x, kind="stable")[:k]
    assert set(np.unique(d)) <= set(top.tolist())
    p = np.zeros(300)
    p[top] = softmax(x[top])
    ok, stat = chi2_ok(np.bincount(d, minlength=300), p, n)
    assert ok, stat


def test_top_p_nucleus():
    x = np.log(np.array([0.5, 0.2, 0.15, 0.1, 0.05], np.float64)).astype(np.float32)
    n = 20000
    # 0.5 + 0.2 + 0.15 = 0.85 >= 0.8: three candidates, renormalised
    d = draws(x, n, temperature=1.0, top_k=0, top_p=0.8, seed=4)
    assert set(np.unique(d)) == {0, 1, 2}
    ok, stat = chi2_ok(np.bincount(d, minlength=5), np.array([0.5, 0.2, 0.15, 0, 0]) / 0.85, n)
    assert ok, stat
    # top_p below the largest probability keeps only the maximum
    assert set(draws(x, 200, temperature=1.0, top_k=0, top_p=0.1, seed=4)) == {0}


def test_repeat_penalty():
    x = np.array([2.0, 2.0, -1.0, 0.5], np.float32)
    n = 20000
    d = draws(x, n, temperature=1.0, top_k=0, top_p=1.0, repeat_penalty=2.0, repeat_last_n=3, seed=11,
              recent=[1, 2, 9, 1])  # 9 is outside the vocabulary; 1 appears twice, penalised once
    pen = np.array([2.0, 1.0, -1.0, 0.5])  # window = the last 3 ids: 2, 9, 1
    pen[2] = -2.0
    ok, stat = chi2_ok(np.bincount(d, minlength=4), softmax(pen), n)
    assert ok, stat
    # the window is the LAST repeat_last_n ids
    assert orl.sample(x, temperature=0, repeat_penalty=2.0, repeat_last_n=1, recent=[0, 1]) == 0
    assert orl.sample(x, temperature=0, repeat_penalty=2.0, repeat_last_n=2, recent=[0, 1]) == 0
    assert orl.sample(x, temperature=0, repeat_penalty=2.0, repeat_last_n=1, recent=[1, 0]) == 1


def test_special_values():
    x = np.array([np.nan, -np.inf, 1.0, np.nan, 1.0], np.float32)
    assert orl.sample(x, temperature=0) == 2
    for kw in (dict(top_k=0, top_p=1.0), dict(top_k=3, top_p=1.0), dict(top_k=0, top_p=0.9)):
        d = set(draws(x, 300, temperature=1.0, seed=1, **kw))
        assert d == {2, 4}, (kw, d)
    # two equal maxima hold half the mass each: top_p 0.5 keeps the first (lower index)
    assert set(draws(x, 300, temperature=1.0, seed=1, top_k=0, top_p=0.5)) == {2}
    assert orl.sample(np.full(10, -np.inf, np.float32), temperature=1.0, top_k=0, top_p=1.0) == 0


@pytest.mark.parametrize("n", [1, 7, 1024, 1025, 50000])
def test_top_k_larger_than_vocab(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    d = draws(x, 50, temperature=0.5, top_k=5000, top_p=1.0, seed=2)
    assert d.min() >= 0 and d.max() < n
