"""GGUF container: the assertions of the reference's gguf/gguf_test.go, against
the product's reader (gb_gguf_*) and the oracle's reader."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _read(name):
    with open(os.path.join(GOLD, name), "rb") as f:
        return f.read()


def test_roundtrip_product_reader(gb):
    # gguf/gguf_test.go:TestRoundTrip (lines 49-97)
    f = gb.Gguf(_read("roundtrip.gguf"))
    version, alignment, n_kv, n_t = f.header()
    assert (version, alignment) == (3, 32)
    assert f.string("general.architecture") == "llama"
    assert f.uint("llama.block_count") == 2
    assert f.float("llama.rope.freq_base") == 10000
    assert f.strings("tokenizer.ggml.tokens") == ["<s>", "</s>", "hello"]
    assert f.floats("tokenizer.ggml.scores") == [0.0, -1.0, 2.5]
    keys = f.keys()
    assert dict(keys)["x.flag"] == 7
    assert np.int64(np.uint64(f.uint("x.big"))) == -7
    assert n_kv == 7 and keys[0][0] == "general.architecture"
    ta = f.tensor("a.weight")
    assert ta["type"] == 0 and ta["bytes"] == 48 and ta["dims"] == [3, 4]
    assert ta["data"] == b"".join(np.arange(12, dtype=np.float32).tobytes() for _ in [0])
    tq = f.tensor("q.weight")
    assert tq["type"] == 8 and tq["bytes"] == 136 and tq["offset"] % 32 == 0
    assert tq["data"] == bytes(i & 0xFF for i in range(136))
    assert f.tensor("nope") is None
    f.close()


def test_roundtrip_oracle_reader(orc):
    import ctypes as C

    g = orc.Gguf(_read("roundtrip.gguf"))
    L = orc.lib()
    assert L.or_gguf_version(g.h) == 3 and L.or_gguf_alignment(g.h) == 32
    assert L.or_gguf_n_kv(g.h) == 7 and L.or_gguf_n_tensors(g.h) == 2
    assert L.or_gguf_uint(g.h, b"llama.block_count", 0) == 2
    assert L.or_gguf_float(g.h, b"llama.rope.freq_base", 0) == 10000
    buf = C.create_string_buffer(64)
    L.or_gguf_string(g.h, b"general.architecture", b"", buf, 64)
    assert buf.value == b"llama"
    g.close()


def test_corrupt_rejected_by_both(gb, orc):
    # gguf/gguf_test.go:TestCorrupt
    good = _read("corrupt_base.gguf")
    gb.Gguf(good).close()
    orc.Gguf(good).close()
    for n in (0, 3, 8, 20, 40, len(good) - 1):
        with pytest.raises(gb.GollamaError):
            gb.Gguf(good[:n])
        with pytest.raises(ValueError):
            orc.Gguf(good[:n])
    bad = b"X" + good[1:]
    with pytest.raises(gb.GollamaError) as e:
        gb.Gguf(bad)
    assert "magic" in str(e.value)
    with pytest.raises(ValueError):
        orc.Gguf(bad)


def test_synth_image_parses_in_both(gb, orc):
    spec = gb.synth_spec(layers=2, dim=256, ffn=512, heads=4, kv_heads=2, vocab=512, ctx_len=64, mix=1, seed=9)
    img = gb.SynthImage(spec)
    data = bytes(img.view())
    f = gb.Gguf(data)
    assert f.uint("llama.block_count") == 2 and f.uint("llama.attention.head_count_kv") == 2
    assert f.tensor("blk.0.attn_v.weight")["type"] == 14  # Q6_K in the Q4_K_M mix
    assert f.tensor("blk.1.ffn_down.weight")["type"] == 12  # odd layers Q4_K
    assert f.tensor("blk.0.ffn_down.weight")["type"] == 14  # even layers Q6_K
    assert f.tensor("output.weight")["type"] == 14
    f.close()
    orc.Gguf(data).close()
