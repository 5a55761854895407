"""The C-ABI boundary without a GPU: the library loads, exports every symbol
include/gollama_b200.h declares, validates like the reference, and its
synthetic-data generators are deterministic."""
import ctypes as C
import os

import numpy as np
import pytest


def test_every_declared_symbol_is_exported(gb):
    lib = gb.lib()
    names = gb.declared_functions()
    assert len(names) > 50
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_error_slot(gb):
    assert b"sm_100a" in gb.lib().gb_version()
    with pytest.raises(gb.GollamaError) as e:
        gb.Gguf(b"")
    assert e.value.code == gb.ERR_IO


def test_host_argmax_rule(gb):
    # model.Argmax, model/model.go:376
    assert gb.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert gb.argmax(np.array([np.nan, 1, 2], np.float32)) == 0
    assert gb.argmax(np.array([0, np.nan, 2], np.float32)) == 2
    assert gb.argmax(np.array([-np.inf, -np.inf], np.float32)) == 0


def test_host_argmax_matches_oracle(gb, orc):
    # the library's two-pass (vectorised) form against the oracle's walk of
    # model.Argmax: ties, NaN at 0 and later, signed zeros, infinities, and
    # lengths around the 16-element blocks
    rng = np.random.default_rng(11)
    specials = np.array([0.0, -0.0, 1.0, -1.0, 3.0, 3.0, np.inf, -np.inf, np.nan, 2.5], np.float32)
    for t in range(3000):
        n = int(rng.integers(1, 80)) if t % 4 else int(rng.integers(1, 5000))
        x = rng.standard_normal(n).astype(np.float32) if t % 3 == 0 else rng.choice(specials, n)
        assert gb.argmax(x) == orc.argmax(x), x
    big = rng.standard_normal(128256).astype(np.float32)
    big[[5, 70000, 128255]] = 9.0  # the first of three equal maxima
    assert gb.argmax(big) == orc.argmax(big) == 5


def test_model_load_rejects_bad_files_without_gpu(gb, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF" + b"\0" * 4)
    with pytest.raises(gb.GollamaError) as e:
        gb.Model(str(p))
    assert e.value.code == gb.ERR_IO
    with pytest.raises(gb.GollamaError):
        gb.Model(str(tmp_path / "missing.gguf"))


def test_synth_matrix_deterministic_across_threads(gb, monkeypatch):
    a = gb.synth_matrix(gb.Q4_K, 64, 1024, seed=5)
    monkeypatch.setenv("GB_HOST_THREADS", "1")
    b = gb.synth_matrix(gb.Q4_K, 64, 1024, seed=5)
    assert a.tobytes() == b.tobytes()
    assert a.tobytes() != gb.synth_matrix(gb.Q4_K, 64, 1024, seed=6).tobytes()


def test_synth_block_recipes(gb, orc):
    # Q4_0: d = |N(0,0.02)|/8 >= 0; Q4_K: d, dmin >= 0; Q6_K: int8 scales in [-32, 31]
    q40 = gb.synth_matrix(gb.Q4_0, 32, 256, seed=1).reshape(-1, 18)
    d = q40[:, :2].copy().view(np.float16).astype(np.float32)
    assert (d >= 0).all() and 0.0005 < float(d.mean()) < 0.005
    q4k = gb.synth_matrix(gb.Q4_K, 32, 256, seed=1).reshape(-1, 144)
    assert (q4k[:, :4].copy().view(np.float16) >= 0).all()
    q6k = gb.synth_matrix(gb.Q6_K, 32, 256, seed=1).reshape(-1, 210)
    sc = q6k[:, 192:208].view(np.int8)
    assert sc.min() >= -32 and sc.max() <= 31
    y = orc.dequantize(gb.Q6_K, q6k.reshape(-1), 32 * 256)
    assert np.isfinite(y).all()


def test_synth_normal_and_kv(gb):
    x = gb.synth_normal(7, 1, 100000)
    assert abs(float(x.mean())) < 0.02 and abs(float(x.std()) - 1) < 0.02
    assert x.tobytes() == gb.synth_normal(7, 1, 100000).tobytes()
    k, v = gb.synth_kv_normal(3, 2, 10, 4, 256, True)
    k2, _ = gb.synth_kv_normal(3, 2, 12, 2, 256, True)
    np.testing.assert_array_equal(k[2:], k2)  # keyed by absolute position
    assert np.array_equal(k, k.astype(np.float16).astype(np.float32))  # rounded through binary16


def test_presets(gb):
    s = gb.synth_preset(8)
    assert (s.layers, s.dim, s.ffn, s.heads, s.kv_heads, s.head_dim, s.vocab) == (32, 4096, 14336, 32, 8, 128, 128256)
    assert s.ctx_len >= 8320
    s1 = gb.synth_preset(1)
    assert s1.mix == 0 and s1.head_dim == 64
    with pytest.raises(gb.GollamaError):
        gb.synth_preset(5)


def test_header_declares_reference_citations():
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                            "gollama_b200.h")).read()
    for cite in ("backend/gpu/gpu.go:35", "backend/gpu/gpu.go:137", "model/model.go:313",
                 "model/model.go:376", "gguf/gguf.go:62"):
        assert cite in hdr
