"""The device sampler (gb_gpu_sample, gb_model_set_sampler) against the host
restatement of its rule (oracle or_sample), token for token: the rule fixes
every float32 operation and the association of every sum, so the two must
pick the same id for every (logits, parameters, context, counter)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [
    dict(temperature=0.0),
    dict(temperature=0.8, top_k=40, top_p=0.95),
    dict(temperature=1.0, top_k=0, top_p=1.0),
    dict(temperature=0.7, top_k=0, top_p=0.9),
    dict(temperature=1.3, top_k=1024, top_p=1.0),
    dict(temperature=0.9, top_k=5000, top_p=0.5),
    dict(temperature=1.0, top_k=1),
    dict(temperature=2.5, top_k=7, top_p=0.3),
    dict(temperature=0.6, top_k=50, top_p=1.0, repeat_penalty=1.3, repeat_last_n=64),
    dict(temperature=0.0, repeat_penalty=1.8, repeat_last_n=200),
    dict(temperature=1.1, top_k=0, top_p=1.0, repeat_penalty=0.7, repeat_last_n=16),
]


def params(gb, seed, **kw):
    base = dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64)
    base.update(kw)
    return gb.sample_params(seed=seed, **base)


def run_gpu(kernels, gb, logits, prm, recent, counter):
    dl = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    rec = np.ascontiguousarray(np.asarray(recent, np.int32))
    dr = torch.from_numpy(rec).cuda() if rec.size else None
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    kernels.sample(dl, logits.size, prm, dr, rec.size, counter, out)
    torch.cuda.synchronize()
    return int(out.item())


@pytest.mark.parametrize("n", [50, 1000, 32000, 128256])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_sample_matches_rule(kernels, gb, orc, cuda, n, ci):
    case = CASES[ci]
    rng = np.random.default_rng(1000 * ci + n)
    logits = (3 * rng.standard_normal(n)).astype(np.float32)
    logits[rng.integers(0, n, 4)] = logits.max()  # tied maxima
    recent = rng.integers(-3, n + 3, 300).astype(np.int32)  # includes ids outside the vocabulary
    prm = params(gb, seed=77 + ci, **case)
    for counter in range(0, 48, 3):
        want = orc.sample(logits, recent=recent, counter=counter, seed=77 + ci,
                          **{**dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64),
                             **case})
        got = run_gpu(kernels, gb, logits, prm, recent, counter)
        assert got == want, f"n={n} case={case} counter={counter}: gpu {got} vs rule {want}"


def test_sample_special_values(kernels, gb, orc, cuda):
    x = np.array([np.nan, -np.inf, 1.0, np.nan, 1.0, -0.0, 0.0] + [-1.0] * 3000, np.float32)
    for case in CASES:
        prm = params(gb, seed=3, **case)
        for counter in range(8):
            want = orc.sample(x, seed=3, counter=counter, recent=[5, 6],
                              **{**dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.0,
                                        repeat_last_n=64), **case})
            assert run_gpu(kernels, gb, x, prm, [5, 6], counter) == want
    allinf = np.full(2000, -np.inf, np.float32)
    assert run_gpu(kernels, gb, allinf, params(gb, 1, temperature=1.0, top_k=0, top_p=1.0), [], 0) == 0
    flat = np.zeros(5000, np.float32)  # every token tied: the candidates are the lowest indices
    for counter in range(8):
        prm = params(gb, 2, temperature=1.0, top_k=100, top_p=1.0)
        want = orc.sample(flat, temperature=1.0, top_k=100, top_p=1.0, seed=2, counter=counter)
        got = run_gpu(kernels, gb, flat, prm, [], counter)
        assert got == want and got < 100


def test_sample_distribution_on_device(kernels, gb, orc, cuda):
    # fixed logits, many counters: the device's draws follow the tempered softmax
    rng = np.random.default_rng(5)
    x = (2 * rng.standard_normal(20)).astype(np.float32)
    prm = params(gb, 9, temperature=0.9, top_k=0, top_p=1.0)
    got = np.bincount([run_gpu(kernels, gb, x, prm, [], c) for c in range(3000)], minlength=20)
    p = np.exp(x / np.float64(0.9) - (x / np.float64(0.9)).max())
    p /= p.sum()
    tv = 0.5 * np.abs(got / got.sum() - p).sum()
    assert tv < 0.05, tv


def test_sample_rejects_bad_arguments(kernels, gb, cuda):
    dl = torch.zeros(10, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    prm = params(gb, 0)
    with pytest.raises(gb.GollamaError):
        kernels.sample(dl, 0, prm, None, 0, 0, out)
    with pytest.raises(gb.GollamaError):
        kernels.sample(dl, (1 << 20) + 1, prm, None, 0, 0, out)


CFG = dict(layers=2, dim=512, ffn=1024, heads=8, kv_heads=2, head_dim=64, vocab=1024, ctx_len=96, mix=1, seed=21)


@pytest.mark.parametrize("graph", [1, 0])
def test_model_sampled_generation_matches_rule(gb, orc, cuda, graph):
    """generate() with a sampler: every token equals the rule applied to the
    step's logits, with the penalty window over the fed tokens (prompt
    included) and counter = position."""
    img = gb.SynthImage(gb.synth_spec(**CFG))
    kw = dict(temperature=0.9, top_k=50, top_p=0.9, repeat_penalty=1.2, repeat_last_n=8)
    prompt = [3, 77, 500, 77, 9]
    n = 12
    m = gb.Model(img, max_len=64, use_graph=graph)
    for p, t in enumerate(prompt[:-1]):
        m.forward(t, p)
    m.set_sampler(gb.sample_params(seed=123, **kw))
    toks = [int(t) for t in m.generate(prompt[-1], len(prompt) - 1, n)]
    m.close()
    # replay: the same logits from the greedy step, the rule on the host
    r = gb.Model(img, max_len=64, use_graph=graph)
    fed = list(prompt)
    for p, t in enumerate(prompt[:-1]):
        r.forward(t, p)
    for i in range(n):
        pos = len(prompt) - 1 + i
        logits = r.forward(fed[-1], pos).copy()
        want = orc.sample(logits, seed=123, counter=pos, recent=fed, **kw)
        assert toks[i] == want, f"step {i}: device {toks[i]} vs rule {want}"
        fed.append(want)
    r.close()


def test_model_temperature_zero_is_greedy(gb, cuda):
    img = gb.SynthImage(gb.synth_spec(**CFG))
    m = gb.Model(img, max_len=64)
    greedy = m.generate(5, 0, 10).copy()
    m.set_sampler(gb.sample_params(temperature=0.0, seed=1))
    same = m.generate(5, 0, 10).copy()
    m.set_sampler(None)
    again = m.generate(5, 0, 10).copy()
    m.close()
    assert list(greedy) == list(same) == list(again)
