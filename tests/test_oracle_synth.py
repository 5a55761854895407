"""The oracle's synthetic-input generator (oracle/synth.c) writes the same
bytes as the product library's (gb_synth_model / gb_synth_kv_normal), so the
reference arm of bench.py and the parity checks can build the benchmark's
models without loading the product library. CPU only."""
import numpy as np
import pytest

SPECS = [
    dict(layers=2, dim=256, ffn=512, heads=4, kv_heads=2, vocab=300, ctx_len=64, mix=m, seed=s)
    for m, s in [(0, 0), (1, 3), (2, 1), (3, 2), (4, 5), (5, 7), (6, 11)]
] + [dict(layers=1, dim=512, ffn=768, heads=8, kv_heads=8, head_dim=128, vocab=1000, ctx_len=96, mix=1, seed=9)]


@pytest.mark.parametrize("kw", SPECS, ids=lambda kw: f"mix{kw['mix']}-seed{kw['seed']}")
def test_images_identical(gb, orc, kw):
    img = gb.SynthImage(gb.synth_spec(**kw))
    want = np.array(img.view(), copy=True)
    img.close()
    got = orc.synth_model(orc.synth_spec(**kw))
    assert got.size == want.size
    assert np.array_equal(got, want)


def test_presets_match(gb, orc):
    for p in (1, 3, 8, 70):
        a, b = gb.synth_preset(p), orc.synth_preset(p)
        for f, _ in orc.SynthSpec._fields_:
            assert getattr(a, f) == getattr(b, f), (p, f)


@pytest.mark.parametrize("f16", [0, 1])
def test_kv_fill_identical(gb, orc, f16):
    for layer, pos0, n in [(0, 0, 100), (3, 8000, 77), (31, 5, 1)]:
        k0, v0 = gb.synth_kv_normal(1, layer, pos0, n, 1024, bool(f16))
        k1, v1 = orc.synth_kv_normal(1, layer, pos0, n, 1024, bool(f16))
        assert np.array_equal(k0.view(np.uint32), k1.view(np.uint32))
        assert np.array_equal(v0.view(np.uint32), v1.view(np.uint32))
