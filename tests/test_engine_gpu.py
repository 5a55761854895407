"""Continuous batching (gb_engine_*; the reference's roadmap "Paged KV cache
plus continuous batching", ROADMAP.md:197-202): sequences that join and leave
between steps are decoded together, one batched pass per step, each through
its own pages of the paged KV pool. Every row's logits must match the same
sequence decoded alone by the one-sequence model (gb_model_forward) and by
cpuForward (model/model_test.go:114, the C oracle) to the prefill's
tolerance: the batched pass uses the binary16-operand tensor-core GEMMs, the
one-sequence decode the float32-exact GEMVs."""
import numpy as np
import pytest

from test_model_gpu import MODELS

pytestmark = pytest.mark.gpu

# relative to the largest |logit|: looser than the prefill-vs-decode bar, as
# here the lm_head too runs on binary16 operands and every position is
# checked (measured on B200: median 2-6e-4, worst 1.4e-2 for single tokens
# whose logits are all small); the isolation check above is the tight one (a wrong
# page or a stale cache row gives errors of order 1)
LOGIT_TOL = 2e-2


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / (np.abs(b).max() + 1e-30))


@pytest.mark.parametrize("name,page", [("q4km_hd64", 16), ("q4km_hd128", 32), ("gqa8_hd128", 8), ("q5km", 16)])
def test_engine_matches_one_sequence_decode(gb, orc, cuda, name, page):
    cfg = MODELS[name]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(7)
    m = gb.Model(img, max_len=96)
    e = gb.Engine(m, page_size=page, n_pages=64, max_batch=8)
    # prompts; C joins at step 4, A leaves after step 14 and D takes its pages
    prompts = {k: [int(t) for t in rng.integers(0, cfg["vocab"], n)] for k, n in (("A", 11), ("B", 19), ("C", 5),
                                                                                  ("D", 9))}
    join = {"A": 0, "B": 0, "C": 4, "D": 15}
    leave = {"A": 14}
    ids, fed, got, nxt_tok = {}, {}, {}, {}
    for step in range(26):
        for k, s0 in join.items():
            if s0 == step:
                ids[k] = e.add()
                fed[k], got[k] = [], []
        live = [k for k in ids if k not in leave or step <= leave[k]]
        toks = []
        for k in live:
            i = len(fed[k])
            toks.append(prompts[k][i] if i < len(prompts[k]) else nxt_tok[k])
        logits, nxt = e.step([ids[k] for k in live], toks)
        for j, k in enumerate(live):
            fed[k].append(toks[j])
            got[k].append(logits[j].copy())
            nxt_tok[k] = int(nxt[j])
            assert nxt[j] == int(np.argmax(logits[j]))  # the first maximum
            assert e.seq_len(ids[k]) == len(fed[k])
        for k, s1 in leave.items():
            if s1 == step:
                before = e.free_pages()
                e.release(ids[k])
                assert e.free_pages() > before
                del ids[k]
    # each sequence alone through the one-sequence decode
    # isolation: each sequence replayed alone (batches of one) in a fresh engine
    # gives the same rows up to the summation order of the attention splits
    m2 = gb.Model(img, max_len=96)
    e2 = gb.Engine(m2, page_size=page, n_pages=64, max_batch=8)
    for k in fed:
        sid = e2.add()
        for p, t in enumerate(fed[k]):
            alone, _ = e2.step([sid], [t])
            assert rel_err(got[k][p], alone[0]) < 1e-4, f"{name} seq {k} pos {p}: batched vs alone"
        e2.release(sid)
    e2.close()
    m2.close()
    # against the one-sequence decode (float32-exact GEMVs)
    errs = []
    for k in fed:
        r = gb.Model(img, max_len=96)
        for p, t in enumerate(fed[k]):
            want = r.forward(t, p)
            errs.append(rel_err(got[k][p], want))
            assert errs[-1] < LOGIT_TOL, f"{name} seq {k} pos {p}: {errs[-1]:.3g}"
        r.close()
    print(f"{name}: {len(errs)} rows, worst {max(errs):.2e}, median {np.median(errs):.2e}")
    # against cpuForward itself (the C restatement, binary16 KV semantics),
    # each sequence on its own oracle: every row within the binary16-GEMM
    # tolerance, and the engine's greedy token equal to model.Argmax of the
    # oracle's logits wherever the oracle's top two are further apart than
    # that tolerance
    raw = np.array(img.view(), copy=True)
    oracle_errs = []
    for k in fed:
        om = orc.OracleModel(raw, 96, True)
        for p, t in enumerate(fed[k]):
            want = om.forward(t, p, cfg["vocab"])
            oracle_errs.append(rel_err(got[k][p], want))
            assert oracle_errs[-1] < LOGIT_TOL, f"{name} seq {k} pos {p} vs oracle: {oracle_errs[-1]:.3g}"
            top = np.sort(want.astype(np.float64))
            if top[-1] - top[-2] > 2 * LOGIT_TOL * np.abs(want).max():
                assert int(np.argmax(got[k][p])) == orc.argmax(want), f"{name} seq {k} pos {p}: greedy token"
        om.close()
    print(f"{name} vs oracle: worst {max(oracle_errs):.2e}, median {np.median(oracle_errs):.2e}")
    e.close()
    m.close()


def test_engine_page_exhaustion_and_errors(gb, cuda):
    cfg = MODELS["q4km_hd64"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    m = gb.Model(img, max_len=96)
    e = gb.Engine(m, page_size=16, n_pages=2, max_batch=4)
    a, b, c = e.add(), e.add(), e.add()
    e.step([a, b], [1, 2])  # one page each
    with pytest.raises(gb.GollamaError) as err:
        e.step([a, b, c], [3, 4, 5])  # c needs a third page
    assert "out of KV pages" in str(err.value)
    assert e.seq_len(a) == 1 and e.seq_len(c) == 0  # nothing changed
    with pytest.raises(gb.GollamaError):
        e.step([a], [cfg["vocab"]])
    e.release(b)
    e.step([a, c], [3, 4])  # c takes b's page
    assert e.free_pages() == 0
    e.close()
    # a sequence listed several times takes that many positions: 97 rows
    # pass the 96-position cache, and nothing changes
    e = gb.Engine(m, page_size=16, n_pages=16, max_batch=128)
    a = e.add()
    with pytest.raises(gb.GollamaError) as err:
        e.step([a] * 97, [1] * 97)
    assert "is full" in str(err.value)
    assert e.seq_len(a) == 0 and e.free_pages() == 16
    e.step([a] * 96, [1] * 96)
    assert e.seq_len(a) == 96 and e.free_pages() == 10
    e.close()
    m.close()


def test_engine_prompt_chunk_in_one_step(gb, cuda):
    # a prompt fed as rows of one step (the batched GEMMs) gives the rows the
    # same logits as feeding it token by token, next to another sequence that
    # decodes one token in the same step; decoding then continues from it
    cfg = MODELS["q4km_hd128"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(21)
    prompt = [int(t) for t in rng.integers(0, cfg["vocab"], 40)]
    other = [int(t) for t in rng.integers(0, cfg["vocab"], 8)]
    m = gb.Model(img, max_len=96)
    e = gb.Engine(m, page_size=16, n_pages=32, max_batch=64)
    a, b = e.add(), e.add()
    for t in other[:4]:
        e.step([b], [t])
    logits, nxt = e.step([a] * len(prompt) + [b], prompt + [other[4]])
    chunk = logits[:len(prompt)].copy()
    assert e.seq_len(a) == len(prompt) and e.seq_len(b) == 5
    cont = [e.step([a], [int(nxt[len(prompt) - 1])])[0][0].copy()]
    e.close()
    # the same prompt token by token in a fresh engine
    e = gb.Engine(m, page_size=16, n_pages=32, max_batch=64)
    a = e.add()
    rows = [e.step([a], [t])[0][0].copy() for t in prompt]
    ref_next = int(np.argmax(rows[-1]))
    cont_ref = e.step([a], [ref_next])[0][0].copy()
    e.close()
    m.close()
    for p in range(len(prompt)):
        assert rel_err(chunk[p], rows[p]) < 1e-3, f"pos {p}: {rel_err(chunk[p], rows[p]):.3g}"
    top = np.sort(rows[-1].astype(np.float64))
    if top[-1] - top[-2] > 2e-3 * np.abs(rows[-1]).max():  # not a near-tie
        assert int(nxt[len(prompt) - 1]) == ref_next
        assert rel_err(cont[0], cont_ref) < 1e-3


def test_engine_f16_weight_copy(gb, cuda):
    # the engine's GEMMs through the model's binary16 weight copy (the
    # few-token kernel: the same binary16 products, float32 sums in another
    # order): every row within float32 accumulation of the decoding GEMM's
    cfg = MODELS["q5km"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(9)
    seqs = [[int(t) for t in rng.integers(0, cfg["vocab"], 12)] for _ in range(5)]
    outs = []
    for cached in (False, True):
        m = gb.Model(img, max_len=96)
        if cached:
            m.cache_f16_weights()
        e = gb.Engine(m, page_size=16, n_pages=64, max_batch=8)
        ids = [e.add() for _ in seqs]
        rows = []
        for p in range(12):
            logits, nxt = e.step(ids, [s[p] for s in seqs])
            rows.append((logits.copy(), nxt.copy()))
        e.close()
        m.close()
        outs.append(rows)
    for (la, na), (lb, nb) in zip(*outs):
        for j in range(len(seqs)):
            assert rel_err(lb[j], la[j]) < 1e-3
            top = np.sort(la[j].astype(np.float64))
            if top[-1] - top[-2] > 2e-3 * np.abs(la[j]).max():
                assert na[j] == nb[j]


def test_engine_long_sequences_split_attention(gb, cuda):
    # sequences past 256 positions: the paged attention splits each (sequence,
    # KV head) and merges the splits into the binary16 input of the o GEMM.
    # Each row must equal the sequence run alone (the batch does not leak
    # between sequences) and stay near the one-sequence decode; that bar is
    # looser than at short lengths because the two paths' binary16 vs exact
    # GEMM differences pass into 300 positions of KV cache.
    cfg = dict(MODELS["q4km_hd64"], ctx_len=512)
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(11)
    lens = (330, 290)
    seqs = [[int(t) for t in rng.integers(0, cfg["vocab"], n)] for n in lens]

    def run(batch):
        m = gb.Model(img, max_len=512)
        e = gb.Engine(m, page_size=32, n_pages=32, max_batch=4)
        got = [[] for _ in seqs]
        for group in ([0, 1],) if batch else ([0], [1]):
            ids = {j: e.add() for j in group}
            for p in range(max(lens[j] for j in group)):
                live = [j for j in group if p < lens[j]]
                logits, _ = e.step([ids[j] for j in live], [seqs[j][p] for j in live])
                for r, j in enumerate(live):
                    got[j].append(logits[r].copy())
            for j in group:
                e.release(ids[j])
        e.close()
        m.close()
        return got

    together, alone = run(True), run(False)
    errs = []
    for j, s in enumerate(seqs):
        r = gb.Model(img, max_len=512)
        for p, t in enumerate(s):
            want = r.forward(t, p)
            assert rel_err(together[j][p], alone[j][p]) < 1e-4, f"seq {j} pos {p}: batched vs alone"
            if p >= 250:
                errs.append(rel_err(together[j][p], want))
        r.close()
    print(f"positions 250+: worst {max(errs):.2e}, median {np.median(errs):.2e}")
    assert max(errs) < 5e-2 and np.median(errs) < 5e-3
