"""The decode step on the GPU against cpuForward (model/model_test.go:114) on the
same seeded synthetic GGUF: logits within 1e-3 abs + 1e-4 rel, identical greedy
tokens, KV caches that match, and the reference's validation errors."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4  # BASELINE parity bound on logits

MODELS = {
    "q4km_hd64": dict(layers=2, dim=512, ffn=1024, heads=8, kv_heads=2, head_dim=64, vocab=1000, ctx_len=96, mix=1, seed=11),
    "q40_tied": dict(layers=2, dim=256, ffn=512, heads=4, kv_heads=2, head_dim=64, vocab=512, ctx_len=96, mix=0, seed=12),
    "q4km_hd128": dict(layers=3, dim=512, ffn=768, heads=4, kv_heads=2, head_dim=128, vocab=777, ctx_len=96, mix=1, seed=13),
    "q4k_all": dict(layers=2, dim=512, ffn=512, heads=4, kv_heads=4, head_dim=128, vocab=600, ctx_len=96, mix=2, seed=14),
    # GQA groups of 3 and 8 query heads per KV head
    "gqa3_hd64": dict(layers=2, dim=768, ffn=512, heads=12, kv_heads=4, head_dim=64, vocab=500, ctx_len=96, mix=1, seed=15),
    "gqa8_hd128": dict(layers=2, dim=1024, ffn=512, heads=8, kv_heads=1, head_dim=128, vocab=500, ctx_len=96, mix=1, seed=16),
    # all Q8_0 (untied head)
    "q80_all": dict(layers=2, dim=512, ffn=768, heads=8, kv_heads=2, head_dim=64, vocab=700, ctx_len=96, mix=4, seed=17),
    # all F16 matrices (model.uploadLinear's F16 case, MatVecF16)
    "f16_all": dict(layers=2, dim=512, ffn=768, heads=8, kv_heads=2, head_dim=64, vocab=700, ctx_len=96, mix=5, seed=18),
    # Q5_K_M mix (Q5_K with Q6_K attn_v, even-layer ffn_down and output; Q5_K embedding)
    "q5km": dict(layers=2, dim=512, ffn=768, heads=8, kv_heads=2, head_dim=128, vocab=900, ctx_len=96, mix=6, seed=19),
}


def make(gb, name):
    spec = gb.synth_spec(**MODELS[name])
    img = gb.SynthImage(spec)
    return img, np.array(img.view(), copy=True)


def kv_report(m, om, orc, cfg, n_pos, kv_f16):
    """Where the KV caches first differ from cpuForward's: localises a logits mismatch."""
    import ctypes as C

    kv_dim = cfg["kv_heads"] * cfg["head_dim"]
    tol = 4e-3 if kv_f16 else 1e-4
    out = []
    for layer in range(cfg["layers"]):
        k, v = m.read_kv(layer, 0, n_pos)
        kp = orc.lib().or_model_kcache(om.h, layer)
        vp = orc.lib().or_model_vcache(om.h, layer)
        kw = np.ctypeslib.as_array((C.c_float * (n_pos * kv_dim)).from_address(kp)).reshape(n_pos, kv_dim)
        vw = np.ctypeslib.as_array((C.c_float * (n_pos * kv_dim)).from_address(vp)).reshape(n_pos, kv_dim)
        for nm, g, w in (("K", k, kw), ("V", v, vw)):
            bad = np.abs(g - w) > tol * (1 + np.abs(w))
            if bad.any():
                p, j = np.argwhere(bad)[0]
                out.append(f"layer {layer} {nm}: {int(bad.sum())} bad, first at pos {p} dim {j}")
    return "; ".join(out) if out else "KV caches match"


def check_logits(name, got, want, report=None):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bad = d > ATOL + RTOL * np.abs(want)
    if bad.any():
        tiles = sorted({int(i) // 32 for i in np.flatnonzero(bad)})
        msg = (f"{name}: max abs diff {d.max():.3g} at {int(np.argmax(d))}; {int(bad.sum())} of {bad.size} "
               f"logits bad, 32-row tiles {tiles[:16]}")
        if report is not None:
            msg += "; " + report()
        raise AssertionError(msg)
    return float(d.max())


def near_tie(logits, tol=1e-3):
    s = np.sort(logits.astype(np.float64))
    return s[-1] - s[-2] < tol


@pytest.mark.parametrize("name", list(MODELS))
@pytest.mark.parametrize("kv_f16", [0, 1])
def test_forward_vs_cpu(gb, orc, cuda, name, kv_f16):
    img, raw = make(gb, name)
    cfg = MODELS[name]
    m = gb.Model(img, max_len=64, kv_f16=kv_f16)
    om = orc.OracleModel(raw, 64, bool(kv_f16))
    rng = np.random.default_rng(cfg["seed"])
    worst = 0.0
    for pos, tok in enumerate(rng.integers(0, cfg["vocab"], 8)):
        got = m.forward(int(tok), pos).copy()
        want = om.forward(int(tok), pos, cfg["vocab"])
        rep = lambda: kv_report(m, om, orc, cfg, pos + 1, kv_f16)
        worst = max(worst, check_logits(f"{name} kv_f16={kv_f16} pos {pos}", got, want, rep))
        if not near_tie(want):
            assert gb.argmax(got) == orc.argmax(want)
    m.close()
    om.close()
    assert worst < ATOL


def test_graph_and_eager_identical(gb, cuda):
    img, _ = make(gb, "q4km_hd64")
    a = gb.Model(img, max_len=64, use_graph=1)
    b = gb.Model(img, max_len=64, use_graph=0)
    for pos, tok in enumerate([5, 17, 999, 0]):
        la = a.forward(tok, pos).copy()
        lb = b.forward(tok, pos).copy()
        assert la.tobytes() == lb.tobytes()
    a.close()
    b.close()


def test_forward_into_page_locked_buffer(gb, cuda):
    # a page-locked caller buffer receives the device copy directly; the same
    # position recomputed into pageable memory (through the staging buffer)
    # gives the same bytes
    img, _ = make(gb, "q4km_hd64")
    m = gb.Model(img, max_len=64)
    pinned = torch.empty(m.config.vocab, dtype=torch.float32, pin_memory=True).numpy()
    pageable = np.empty(m.config.vocab, np.float32)
    for pos, tok in enumerate([5, 17, 999]):
        m.forward(tok, pos, out=pinned)
        m.forward(tok, pos, out=pageable)
        assert pinned.tobytes() == pageable.tobytes()
    m.close()


@pytest.mark.parametrize("name", ["q4km_hd64", "q40_tied", "q4km_hd128"])
def test_greedy_generation_matches_cpu(gb, orc, cuda, name):
    # cmd/gollama/run.go:110-136: prompt fed one token at a time, then greedy
    img, raw = make(gb, name)
    cfg = MODELS[name]
    m = gb.Model(img, max_len=64)
    om = orc.OracleModel(raw, 64, True)
    prompt = [3, 141, 59, 26]
    for pos, tok in enumerate(prompt):
        m.forward(tok, pos)
        want = om.forward(tok, pos, cfg["vocab"])
    nxt = orc.argmax(want)
    gen_gpu = m.generate(nxt, len(prompt), 12)
    toks, t = [], nxt
    for i in range(12):
        logits = om.forward(t, len(prompt) + i, cfg["vocab"])
        if near_tie(logits):
            break  # a logit near-tie may legitimately differ
        t = orc.argmax(logits)
        toks.append(t)
    assert list(gen_gpu[:len(toks)]) == toks
    # the device greedy step agrees with the host Argmax of Forward's logits
    lg = m.forward(int(gen_gpu[0]), len(prompt) + 1).copy()
    assert m.next(int(gen_gpu[0]), len(prompt) + 1) == gb.argmax(lg)
    m.close()
    om.close()


@pytest.mark.parametrize("kv_f16", [0, 1])
def test_kv_cache_matches_cpu(gb, orc, cuda, kv_f16):
    import ctypes as C

    img, raw = make(gb, "q4km_hd128")
    cfg = MODELS["q4km_hd128"]
    m = gb.Model(img, max_len=64, kv_f16=kv_f16)
    om = orc.OracleModel(raw, 64, bool(kv_f16))
    for pos, tok in enumerate([1, 2, 3, 4, 5]):
        m.forward(tok, pos)
        om.forward(tok, pos, cfg["vocab"])
    kv_dim = cfg["kv_heads"] * cfg["head_dim"]
    tol = 4e-3 if kv_f16 else 1e-4
    for layer in range(cfg["layers"]):
        k, v = m.read_kv(layer, 0, 5)
        kp = orc.lib().or_model_kcache(om.h, layer)
        vp = orc.lib().or_model_vcache(om.h, layer)
        kw = np.ctypeslib.as_array((C.c_float * (5 * kv_dim)).from_address(kp)).reshape(5, kv_dim)
        vw = np.ctypeslib.as_array((C.c_float * (5 * kv_dim)).from_address(vp)).reshape(5, kv_dim)
        np.testing.assert_allclose(k, kw, atol=tol, rtol=tol)
        np.testing.assert_allclose(v, vw, atol=tol, rtol=tol)
    m.close()
    om.close()


def test_forward_validation(gb, cuda):
    # model/model.go:315-320
    img, _ = make(gb, "q40_tied")
    m = gb.Model(img, max_len=16)
    with pytest.raises(gb.GollamaError) as e:
        m.forward(1, 16)
    assert "position 16 outside the 16-token cache" in str(e.value)
    with pytest.raises(gb.GollamaError) as e:
        m.forward(512, 0)
    assert "token 512 outside the vocabulary" in str(e.value)
    with pytest.raises(gb.GollamaError):
        m.forward(-1, 0)
    m.forward(0, 0)  # still usable
    assert m.config.max_len == 16
    m.close()


def test_max_len_clamps_to_context(gb, cuda):
    # model/model.go:165: maxLen <= 0 or above the context -> context_length
    img, _ = make(gb, "q40_tied")
    for req, want in ((0, 96), (500, 96), (32, 32)):
        m = gb.Model(img, max_len=req)
        assert m.config.max_len == want
        m.close()


def test_prefilled_kv_long_context(gb, orc, cuda):
    # config-4 style: KV prefilled with seeded N(0,1) fp16, decode after it
    cfg = dict(MODELS["q4km_hd128"], ctx_len=1100)
    spec = gb.synth_spec(**cfg)
    img = gb.SynthImage(spec)
    raw = np.array(img.view(), copy=True)
    n_pos = 1000
    m = gb.Model(img, max_len=1100, kv_f16=1)
    m.fill_kv_normal(99, n_pos)
    om = orc.OracleModel(raw, 1100, True)
    kv_dim = cfg["kv_heads"] * cfg["head_dim"]
    for layer in range(cfg["layers"]):
        k, v = gb.synth_kv_normal(99, layer, 0, n_pos, kv_dim, True)
        om.set_kv(layer, 0, k, v)
    kk, vv = m.read_kv(1, 0, n_pos)
    k1, v1 = gb.synth_kv_normal(99, 1, 0, n_pos, kv_dim, True)
    assert kk.tobytes() == k1.tobytes() and vv.tobytes() == v1.tobytes()
    for i, tok in enumerate([7, 8, 9]):
        got = m.forward(tok, n_pos + i).copy()
        want = om.forward(tok, n_pos + i, cfg["vocab"])
        check_logits(f"long pos {n_pos + i}", got, want)
    m.close()
    om.close()


@pytest.mark.parametrize("name,max_len", [("q4km_hd128", 16384), ("q4km_hd64", 16384), ("q4km_hd128", 16376)])
def test_long_context_tensor_map_attention(gb, orc, cuda, name, max_len):
    # fp16 caches with max_len a multiple of 32 move whole 128-position
    # sub-chunks of K and V with one TMA tensor copy each (16376: per-chunk
    # copies only); ~200+ positions per slice so most sub-chunks are whole
    cfg = dict(MODELS[name], ctx_len=max_len)
    spec = gb.synth_spec(**cfg)
    img = gb.SynthImage(spec)
    raw = np.array(img.view(), copy=True)
    n_pos = 16000
    m = gb.Model(img, max_len=max_len, kv_f16=1)
    m.fill_kv_normal(5, n_pos)
    om = orc.OracleModel(raw, max_len, True)
    kv_dim = cfg["kv_heads"] * cfg["head_dim"]
    for layer in range(cfg["layers"]):
        k, v = gb.synth_kv_normal(5, layer, 0, n_pos, kv_dim, True)
        om.set_kv(layer, 0, k, v)
    for i, tok in enumerate([11, 22, 33]):
        got = m.forward(tok, n_pos + i).copy()
        want = om.forward(tok, n_pos + i, cfg["vocab"])
        check_logits(f"{name} max_len {max_len} pos {n_pos + i}", got, want)
    m.close()
    om.close()


@pytest.mark.parametrize("kv_f16", [0, 1])
def test_early_positions_many_slices(gb, orc, cuda, kv_f16):
    # a long cache split into more slices than there are positions yet:
    # the empty slices must drop out of the merge
    cfg = dict(MODELS["gqa3_hd64"], ctx_len=2500)
    spec = gb.synth_spec(**cfg)
    img = gb.SynthImage(spec)
    raw = np.array(img.view(), copy=True)
    m = gb.Model(img, max_len=2500, kv_f16=kv_f16)
    om = orc.OracleModel(raw, 2500, bool(kv_f16))
    for pos, tok in enumerate([3, 1, 4, 1, 5]):
        got = m.forward(tok, pos).copy()
        want = om.forward(tok, pos, cfg["vocab"])
        check_logits(f"early pos {pos}", got, want)
    m.close()
    om.close()


def test_load_from_file(gb, orc, cuda, tmp_path):
    spec = gb.synth_spec(**MODELS["q40_tied"])
    path = str(tmp_path / "m.gguf")
    gb._check(gb.lib().gb_synth_model_file(gb.C.byref(spec), path.encode()))
    m = gb.Model(path, max_len=32)
    raw = np.fromfile(path, np.uint8)
    om = orc.OracleModel(raw, 32, True)
    got = m.forward(5, 0).copy()
    check_logits("file", got, om.forward(5, 0, MODELS["q40_tied"]["vocab"]))
    m.close()
    om.close()


def test_profile_and_bytes(gb, cuda):
    img, _ = make(gb, "q4km_hd64")
    m = gb.Model(img, max_len=64)
    prof = m.profile_step(3, 0)
    assert prof["gate_up"][1] == MODELS["q4km_hd64"]["layers"]
    assert all(v[0] >= 0 for v in prof.values())
    b, g = m.step_bytes(10)
    assert b > g > 0
    assert m.launches_per_step() == 1 + 5 * 2 + 2
    m.close()


def test_config1_baseline_model_prefix(gb, orc, cuda):
    # Llama-3.2-1B shape, Q4_0, tied head, f32 KV, ctx 512
    spec = gb.synth_preset(1)
    img = gb.SynthImage(spec)
    raw = np.array(img.view(), copy=True)
    m = gb.Model(img, max_len=512, kv_f16=0)
    om = orc.OracleModel(raw, 512, False)
    rng = np.random.default_rng(0)
    for pos, tok in enumerate(rng.integers(0, spec.vocab, 3)):
        got = m.forward(int(tok), pos).copy()
        want = om.forward(int(tok), pos, spec.vocab)
        check_logits(f"1B pos {pos}", got, want)
        if not near_tie(want):
            assert gb.argmax(got) == orc.argmax(want)
    m.close()
    om.close()
