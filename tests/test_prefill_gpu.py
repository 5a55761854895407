"""Batched prefill (the reference's roadmap item, ROADMAP.md:36-41, its proof
`TestPrefillVsDecode`) and its tensor-core GEMM.

The GEMM is checked against a float64 product of the same binary16 operands
(x rounded to binary16; W = the oracle's float32 dequantization rounded to
binary16), so only the float32 accumulation order may differ. The model's
prefill is checked against T decode steps: its arithmetic is binary16 operands
with float32 accumulation where the decode path keeps float32-exact integer
dot products, so the KV cache and the logits agree to the tolerances stated
below rather than bit for bit."""
import numpy as np
import pytest
import torch

from test_kernels_gpu import BF16, F16, F32, Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, rand_quant
from test_model_gpu import MODELS

pytestmark = pytest.mark.gpu


def weight_bytes(rng, typ, rows, cols):
    if typ in (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K):
        return rand_quant(rng, typ, rows, cols)
    vals = rng.standard_normal(rows * cols) * 0.05
    if typ == BF16:
        return (vals.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    return (vals.astype(np.float16) if typ == F16 else vals.astype(np.float32)).view(np.uint8)


@pytest.mark.parametrize("rows,cols,T", [(128, 256, 1), (300, 1024, 77), (1000, 4096, 128), (4096, 4096, 300),
                                         (256, 512, 512)])
@pytest.mark.parametrize("typ", [Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32])
def test_matmul_f16_vs_reference(gb, orc, cuda, typ, rows, cols, T):
    rng = np.random.default_rng(rows + cols + T + typ)
    w = weight_bytes(rng, typ, rows, cols)
    w16 = orc.dequantize(typ, w, rows * cols).reshape(rows, cols).astype(np.float16)
    x16 = rng.standard_normal((T, cols)).astype(np.float16)
    want = x16.astype(np.float64) @ w16.astype(np.float64).T
    bound = np.abs(x16.astype(np.float64)) @ np.abs(w16.astype(np.float64)).T
    lin = gb.Linear(typ, w, rows, cols)
    dx = torch.from_numpy(x16.view(np.uint16).copy()).cuda()
    dy = torch.full((T, rows), float("nan"), device="cuda")
    lin.matmul_f16(dx, T, dy)
    torch.cuda.synchronize()
    got = dy.cpu().numpy().astype(np.float64)
    lin.close()
    # float32 accumulation of cols products: well inside cols * 2^-24 of the sum of magnitudes
    err = np.abs(got - want) / (bound * 2.0**-18 + 1e-30)
    assert np.isfinite(got).all(), "rows left unwritten or non-finite"
    assert err.max() <= 1.0, f"worst {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"


def read_kv(m, cfg, n):
    return [m.read_kv(l, 0, n) for l in range(cfg["layers"])]


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / (np.abs(b).max() + 1e-30))


def rms_err(a, b):
    d = np.asarray(a, np.float64) - b
    return float(np.sqrt((d * d).mean()) / (np.sqrt((np.asarray(b, np.float64) ** 2).mean()) + 1e-30))


# Prefill (binary16 GEMM operands, float32 sums) vs decode (float32-exact dot
# products), measured on B200: layer-0 K/V agree to ~5e-4 of the largest
# magnitude (binary16 rounding of x and W); deeper layers to ~5e-3 RMS, with
# single tokens up to ~4e-2 where a sharp attention softmax amplifies the
# rounding of q and k; logits to <= 6e-4 of the largest logit.
KV_RMS_TOL, KV_MAX_TOL, LOGIT_TOL = 1e-2, 1e-1, 5e-3


def check_kv(kv_got, kv_want, what=""):
    for l, ((kg, vg), (kw, vw)) in enumerate(zip(kv_got, kv_want)):
        for nm, g, w in (("K", kg, kw), ("V", vg, vw)):
            assert rms_err(g, w) < KV_RMS_TOL and rel_err(g, w) < KV_MAX_TOL, \
                f"{what} layer {l} {nm}: rms {rms_err(g, w):.3g} max {rel_err(g, w):.3g}"


@pytest.mark.parametrize("name", ["q4km_hd64", "q40_tied", "q4km_hd128", "q4k_all", "gqa3_hd64", "gqa8_hd128",
                                  "q80_all", "f16_all", "q5km"])
@pytest.mark.parametrize("n", [2, 37])
def test_prefill_vs_decode(gb, cuda, name, n):
    cfg = MODELS[name]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(n)
    toks = rng.integers(0, cfg["vocab"], n).astype(np.int32)
    d = gb.Model(img, max_len=64)
    for p, t in enumerate(toks):
        want = d.forward(int(t), p).copy()
    kv_want = read_kv(d, cfg, n)
    d.close()
    m = gb.Model(img, max_len=64)
    got = m.prefill(toks, 0).copy()
    kv_got = read_kv(m, cfg, n)
    m.close()
    check_kv(kv_got, kv_want, name)
    e = rel_err(got, want)
    assert e < LOGIT_TOL, f"logits {e:.3g}"
    print(f"{name} n={n}: logits rel err {e:.2e}")


def test_prefill_long_chunks_and_f32_cache(gb, cuda):
    # more than one 512-token chunk, a prompt not at position 0, the float32 cache
    cfg = dict(MODELS["q4km_hd64"], ctx_len=1400)
    img = gb.SynthImage(gb.synth_spec(**cfg))
    rng = np.random.default_rng(3)
    toks = rng.integers(0, cfg["vocab"], 1100).astype(np.int32)
    for kv_f16 in (1, 0):
        d = gb.Model(img, max_len=1400, kv_f16=kv_f16)
        for p, t in enumerate(toks[:5]):
            d.forward(int(t), p)
        m = gb.Model(img, max_len=1400, kv_f16=kv_f16)
        m.prefill(toks[:5], 0)
        for p, t in enumerate(toks[5:], start=5):
            want = d.forward(int(t), p)
        got = m.prefill(toks[5:], 5)
        assert rel_err(got, want) < LOGIT_TOL, (kv_f16, rel_err(got, want))
        check_kv(read_kv(m, cfg, 1100), read_kv(d, cfg, 1100), f"kv_f16={kv_f16}")
        d.close()
        m.close()


def test_prefill_single_token_is_forward(gb, cuda):
    cfg = MODELS["q4km_hd128"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    m = gb.Model(img, max_len=64)
    a = m.prefill([17], 0).copy()
    b = m.forward(17, 0).copy()
    m.close()
    assert np.array_equal(a, b)


def test_prefill_then_generate(gb, cuda):
    # prefill fills the cache the decode steps read: generation continues from it
    cfg = MODELS["q4km_hd64"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    toks = [5, 99, 300, 7, 42, 1, 0, 999]
    m = gb.Model(img, max_len=64)
    logits = m.prefill(toks, 0)
    first = int(np.argmax(logits))
    out = m.generate(first, len(toks), 6)
    m.close()
    assert len(out) == 6 and (out >= 0).all() and (out < cfg["vocab"]).all()


def test_prefill_rejects_bad_arguments(gb, cuda):
    cfg = MODELS["q40_tied"]
    img = gb.SynthImage(gb.synth_spec(**cfg))
    m = gb.Model(img, max_len=64)
    with pytest.raises(gb.GollamaError):
        m.prefill(np.zeros(65, np.int32), 0)
    with pytest.raises(gb.GollamaError):
        m.prefill([1, cfg["vocab"]], 0)
    with pytest.raises(gb.GollamaError):
        m.prefill(np.zeros(10, np.int32), 60)
    m.close()


@pytest.mark.parametrize("rows,cols,T", [(128, 256, 1), (300, 1024, 77), (1000, 4096, 128), (4096, 4096, 300),
                                         (256, 512, 512), (4096, 14336, 8)])
@pytest.mark.parametrize("typ", [Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32])
def test_matmul_f16_weight_copy(gb, orc, cuda, typ, rows, cols, T):
    # The binary16 weight copy holds the values the decoding GEMM produces, so
    # the GEMMs over it multiply the same binary16 products; they run other
    # kernel shapes (256 weight rows per CTA above 128 token rows, tokens as
    # the MMA's N below) and so other K splits: float32 sums in another
    # order, held to the float32-accumulation bound against the float64
    # product, like the decoding GEMM itself.
    rng = np.random.default_rng(rows * 7 + cols + T + typ)
    w = weight_bytes(rng, typ, rows, cols)
    x16 = rng.standard_normal((T, cols)).astype(np.float16)
    dx = torch.from_numpy(x16.view(np.uint16).copy()).cuda()
    lin = gb.Linear(typ, w, rows, cols)
    n = lin.cache_f16_weights()
    assert n == ((rows + 127) // 128) * 128 * cols * 2
    got = torch.full((T, rows), float("nan"), device="cuda")
    lin.matmul_f16(dx, T, got)
    torch.cuda.synchronize()
    lin.close()
    assert torch.isfinite(got).all()
    w16 = orc.dequantize(typ, w, rows * cols).reshape(rows, cols).astype(np.float16).astype(np.float64)
    ref = x16.astype(np.float64) @ w16.T
    bound = np.abs(x16.astype(np.float64)) @ np.abs(w16).T
    err = np.abs(got.cpu().numpy().astype(np.float64) - ref) / (bound * 2.0**-18 + 1e-30)
    assert err.max() <= 1.0, f"worst {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"


@pytest.mark.parametrize("name", ["q4km_hd64", "q40_tied", "q4k_all", "q80_all", "f16_all", "q5km"])
def test_prefill_f16_weight_copy(gb, cuda, name):
    # prefill through the model's binary16 weight copy, at 199 batched tokens
    # (256-row CTAs) and at 60 (the few-token kernel): the same binary16
    # products as the decoding GEMM with float32 sums in another order, so
    # logits and KV cache within float32 accumulation of it
    cfg = dict(MODELS[name], ctx_len=256)
    img = gb.SynthImage(gb.synth_spec(**cfg))
    for n in (200, 61):
        toks = np.random.default_rng(5 + n).integers(0, cfg["vocab"], n).astype(np.int32)
        a = gb.Model(img, max_len=256)
        want = a.prefill(toks, 0).copy()
        kv_want = read_kv(a, cfg, n)
        a.close()
        b = gb.Model(img, max_len=256)
        assert b.cache_f16_weights() > 0
        assert b.cache_f16_weights() == 0  # already there
        got = b.prefill(toks, 0).copy()
        kv_got = read_kv(b, cfg, n)
        b.close()
        assert rel_err(got, want) < 1e-3, (n, rel_err(got, want))
        for (kg, vg), (kw, vw) in zip(kv_got, kv_want):
            for g_, w_ in ((kg, kw), (vg, vw)):
                assert rms_err(g_, w_) < 1e-3 and rel_err(g_, w_) < 1e-2
