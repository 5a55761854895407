"""Every kernel of the B200 path against the CPU oracle, on the shapes and with
the tolerances of the reference's backend/gpu/gpu_test.go (seeded random data),
plus the tiled GEMV of the model path and the bit-exact dequantization."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F32, F16, BF16 = 2, 8, 12, 13, 14, 0, 1, 30


def randf(rng, n, scale):
    # backend/gpu/gpu_test.go:65 randf: uniform in [-scale, scale)
    return ((rng.random(n, dtype=np.float32) * 2 - 1) * scale).astype(np.float32)


def assert_close(name, got, want, atol, rtol):
    # backend/gpu/gpu_test.go:74 assertClose
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, name
    d = np.abs(got - want)
    bad = (d > atol + rtol * np.abs(want)) | np.isnan(got)
    assert not bad.any(), f"{name}[{np.argmax(bad)}] = {got[np.argmax(bad)]}, want {want[np.argmax(bad)]}"
    return float(d.max()) if d.size else 0.0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rand_quant(rng, typ, rows, cols):
    # backend/gpu/gpu_test.go:221 randQuant: random bytes, scale fields overwritten
    ts, bs = {Q4_0: (18, 32), Q8_0: (34, 32), Q4_K: (144, 256), Q5_K: (176, 256), Q6_K: (210, 256)}[typ]
    w = rng.integers(0, 256, rows * cols // bs * ts, dtype=np.uint8)

    def scale(off, mag):
        n = len(w) // ts
        h = ((rng.random(n) * 2 - 1) * mag).astype(np.float16).view(np.uint8).reshape(n, 2)
        wv = w.reshape(n, ts)
        wv[:, off:off + 2] = h

    if typ == Q4_0:
        scale(0, 0.02)
    elif typ == Q8_0:  # not in randQuant (the reference has no Q8_0 GPU kernel); same recipe
        scale(0, 0.002)
    elif typ in (Q4_K, Q5_K):  # Q5_K: not in randQuant (no reference kernel); the Q4_K recipe
        scale(0, 0.002)
        scale(2, 0.002)
    else:
        scale(208, 0.001)
    return w


def test_load(kernels):
    assert len(kernels) == 11


@pytest.mark.parametrize("rows", [7, 1024])
def test_rmsnorm(kernels, orc, rows):
    rng = np.random.default_rng(1)
    n = 2048
    x, w = randf(rng, rows * n, 3), randf(rng, n, 1)
    want = orc.rmsnorm(x, w, rows, n, 1e-5)
    dx, dw, dout = dev(x), dev(w), torch.zeros(rows * n, device="cuda")
    kernels.rms_norm(dx, dw, dout, rows, n, 1e-5)
    assert_close("RMSNorm", host(dout), want, 1e-5, 1e-4)
    kernels.rms_norm(dx, dw, dx, rows, n, 1e-5)  # in place
    assert_close("RMSNorm(in place)", host(dx), want, 1e-5, 1e-4)


@pytest.mark.parametrize("n", [1, 31, 256, 1000, 32000])
def test_softmax(kernels, orc, n):
    rng = np.random.default_rng(2)
    rows = 3
    x = randf(rng, rows * n, 10)
    want = orc.softmax(x, rows, n)
    dx = dev(x)
    kernels.softmax(dx, dx, rows, n)
    got = host(dx)
    assert_close("Softmax", got, want, 1e-7, 1e-4)
    assert np.all(np.abs(got.reshape(rows, n).astype(np.float64).sum(1) - 1) < 1e-4)


def test_elementwise(kernels, orc):
    rng = np.random.default_rng(3)
    n = 5632 * 4 + 13
    a, b = randf(rng, n, 8), randf(rng, n, 8)
    da, db, dout = dev(a), dev(b), torch.zeros(n, device="cuda")
    kernels.silu_mul(da, db, dout, n)
    assert_close("SiluMul", host(dout), orc.silu_mul(a, b), 1e-5, 1e-5)
    kernels.add(da, db, dout, n)
    assert_close("Add", host(dout), orc.add(a, b), 0, 0)


def test_rope(kernels, orc):
    rng = np.random.default_rng(4)
    rows, nh, hd = 5, 4, 64
    x = randf(rng, rows * nh * hd, 2)
    pos = np.array([0, 1, 2, 1000, 4095], np.int32)
    freq = 1 + 4 * np.abs(randf(rng, hd // 2, 1))
    want = orc.rope(x, pos, freq, rows, nh, hd, 10000.0)
    dx, dpos, dfreq = dev(x), dev(pos), dev(freq)
    kernels.rope(dx, dpos, dfreq, rows, nh, hd, 10000.0)
    # the reference allows 1e-3 (libdevice sincos); float64 angles here meet 1e-6
    assert_close("RoPE", host(dx), want, 1e-6, 1e-6)
    want = orc.rope(x, pos, None, rows, nh, hd, 10000.0)
    ones = torch.ones(hd // 2, device="cuda")
    dx = dev(x)
    kernels.rope(dx, dpos, ones, rows, nh, hd, 10000.0)
    assert_close("RoPE(no factors)", host(dx), want, 1e-6, 1e-6)


def test_matvec_dense(kernels, orc):
    rng = np.random.default_rng(5)
    rows, cols, batch = 300, 2048, 3
    w, x = randf(rng, rows * cols, 0.05), randf(rng, batch * cols, 1)
    hw = w.astype(np.float16)
    w = hw.astype(np.float32)
    want = orc.matvec_f16(hw.view(np.uint16), x, rows, cols, batch)
    dw, dx, dy = dev(hw.view(np.int16)), dev(x), torch.zeros(batch * rows, device="cuda")
    kernels.matvec_f16(dw, dx, dy, rows, cols, batch)
    assert_close("MatVecF16", host(dy), want, 1e-4, 1e-4)
    want = orc.matvec_f32(w, x, rows, cols, batch)
    kernels.matvec_f32(dev(w), dx, dy, rows, cols, batch)
    assert_close("MatVecF32", host(dy), want, 1e-4, 1e-4)


@pytest.mark.parametrize("cols", [1024, 4096])
@pytest.mark.parametrize("typ", [Q4_0, Q4_K, Q6_K])
def test_matvec_quant_raw(kernels, orc, cols, typ):
    # backend/gpu/gpu_test.go:243 TestMatVecQuant
    rng = np.random.default_rng(6 + cols + typ)
    rows, batch = 300, 2
    x = randf(rng, batch * cols, 1)
    w = rand_quant(rng, typ, rows, cols)
    want = orc.matvec_q(typ, w, x, rows, cols, batch)
    dy = torch.zeros(batch * rows, device="cuda")
    kernels.matvec_q(typ, dev(w), dev(x), dy, rows, cols, batch)
    assert_close(f"MatVec{typ}", host(dy), want, 1e-4, 1e-4)


def test_matvec_quant_errors(kernels, gb):
    y = torch.zeros(8, device="cuda")
    with pytest.raises(gb.GollamaError) as e:
        kernels.matvec_q(F32, y, y, y, 8, 8, 1)
    assert "no matvec kernel for F32" in str(e.value)
    with pytest.raises(gb.GollamaError) as e:
        kernels.matvec_q(Q4_K, y, y, y, 8, 100, 1)
    assert "not a multiple of the block (256)" in str(e.value)


# ---- the tiled GEMV of the model path (limb pack + dp4a + TMA bulk staging)
TILED_SHAPES = [(64, 256), (300, 1024), (300, 4096), (4096, 4096), (1000, 14336), (128256, 2048)]


@pytest.mark.parametrize("rows,cols", TILED_SHAPES)
@pytest.mark.parametrize("typ", [Q4_0, Q8_0, Q4_K, Q5_K, Q6_K])
def test_linear_tiled_vs_oracle(gb, orc, cuda, typ, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + typ)
    w = rand_quant(rng, typ, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    want = orc.matvec_q(typ, w, x, rows, cols)
    lin = gb.Linear(typ, w, rows, cols)
    dy = torch.zeros(rows, device="cuda")
    for _ in range(2):  # the second launch reuses the stream-K counters
        lin.matvec(dev(x), dy)
    worst = assert_close(f"Linear[{typ}] {rows}x{cols}", host(dy), want, 1e-4, 1e-4)
    lin.close()
    assert worst < 1e-3


@pytest.mark.parametrize("rows,cols", [(64, 256), (300, 1024), (1000, 4096), (4096, 4096)])
@pytest.mark.parametrize("typ", [F16, BF16, F32])
def test_linear_unquantized_vs_oracle(gb, orc, cuda, typ, rows, cols):
    # model.uploadLinear keeps F16 / F32 matrices (model/model.go:86-96); MatVecF16/F32.
    # BF16 (added) is the top half of a float32.
    rng = np.random.default_rng(rows * 11 + cols + typ)
    vals = rng.standard_normal(rows * cols) * 0.05
    if typ == BF16:
        w = (vals.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    else:
        w = (vals.astype(np.float16) if typ == F16 else vals.astype(np.float32)).view(np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    want = orc.matvec_q(typ, w, x, rows, cols)
    lin = gb.Linear(typ, w, rows, cols)
    dy = torch.zeros(rows, device="cuda")
    for _ in range(2):
        lin.matvec(dev(x), dy)
    assert_close(f"Linear[{typ}] {rows}x{cols}", host(dy), want, 1e-4, 1e-4)
    lin.close()


LIMB_EPS = 0.5 / 127 / 254**2  # half a unit of the last activation limb, per block maximum (about 2^-24)


@pytest.mark.parametrize("ratio", [10.0, 30.0, 1e3, 1e4])
@pytest.mark.parametrize("typ", [Q4_0, Q8_0, Q4_K, Q5_K, Q6_K])
def test_linear_tiled_outlier_activations(gb, orc, cuda, typ, ratio):
    # Heavy-tailed input: in 12 of the 16 256-element blocks one element is
    # `ratio` times the rest (an outlier feature). The staged activation keeps
    # every element to within LIMB_EPS of its block's largest magnitude (plus
    # float32 rounding of the element itself), so row r of the product is
    # within sum_b LIMB_EPS * max_b|x| * sum_{i in b} |W[r,i]| of the exact
    # one: the bound is checked for every row. Up to 30x outliers the rows
    # also meet the reference's MatVecQ tolerance (1e-4 abs + 1e-4 rel); at
    # 100x and beyond rows whose sum cancels can exceed it (the bound holds).
    rows, cols = 300, 4096
    rng = np.random.default_rng(int(ratio) + typ)
    w = rand_quant(rng, typ, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    blocks = np.arange(cols // 256)[rng.permutation(cols // 256)[:12]]
    x[blocks * 256 + rng.integers(0, 256, blocks.size)] *= np.float32(ratio)
    want = orc.matvec_q(typ, w, x, rows, cols)
    lin = gb.Linear(typ, w, rows, cols)
    dy = torch.zeros(rows, device="cuda")
    lin.matvec(dev(x), dy)
    got = host(dy).astype(np.float64)
    lin.close()
    W = np.abs(orc.dequantize(typ, w, rows * cols).reshape(rows, cols // 256, 256).astype(np.float64))
    bmax = np.abs(x.reshape(-1, 256)).max(1).astype(np.float64)
    absx = np.abs(x.astype(np.float64)).reshape(-1, 256)
    bound = (LIMB_EPS * (W.sum(2) * bmax).sum(1) + 2.0 ** -21 * (W * absx).sum((1, 2)) + 1e-6)
    err = np.abs(got - want)
    assert (err <= bound).all(), f"row {int(np.argmax(err / bound))}: error {err.max():.3g} above the limb bound"
    if ratio <= 30:
        assert_close(f"Linear[{typ}] outliers x{ratio:g}", got, want, 1e-4, 1e-4)


@pytest.mark.parametrize("typ", [Q4_0, Q4_K, Q6_K])
def test_linear_tiled_synthetic_recipe(gb, orc, cuda, typ):
    # the BASELINE GEMV-sweep block recipe, one of its shapes
    rows, cols = 4096, 4096
    w = gb.synth_matrix(typ, rows, cols, seed=0)
    x = gb.synth_normal(0, 1, cols)
    want = orc.matvec_q(typ, w, x, rows, cols)
    lin = gb.Linear(typ, w, rows, cols)
    dy = torch.zeros(rows, device="cuda")
    lin.matvec(dev(x), dy)
    assert_close("Linear(synthetic)", host(dy), want, 1e-4, 1e-4)
    lin.close()


@pytest.mark.parametrize("typ,cols", [(Q4_0, 512), (Q8_0, 512), (Q4_K, 1024), (Q5_K, 1024), (Q6_K, 1024), (F16, 64)])
def test_dequant_rows_bit_exact(kernels, orc, typ, cols):
    rng = np.random.default_rng(typ)
    rows = 40
    if typ == F16:
        w = rng.standard_normal(rows * cols).astype(np.float16).view(np.uint8)
    elif typ == Q8_0:
        w = rng.integers(0, 256, rows * cols // 32 * 34, dtype=np.uint8)
        w.reshape(-1, 34)[:, :2] = rng.normal(0, 0.01, (rows * cols // 32, 1)).astype(np.float16).view(np.uint8)
    else:
        w = rand_quant(rng, typ, rows, cols)
    out = torch.zeros(10 * cols, device="cuda")
    kernels.dequant_rows(typ, dev(w), rows, cols, 7, 10, out)
    got = host(out)
    rb = len(w) // rows
    want = np.concatenate([orc.dequantize(typ, w[r * rb:(r + 1) * rb], cols) for r in range(7, 17)])
    assert got.tobytes() == want.tobytes()


def test_dequant_golden_bit_exact(kernels, golden):
    for key, typ, n in (("q4_k", Q4_K, 256), ("q6_k", Q6_K, 256), ("q4_0", Q4_0, 32), ("q8_0", Q8_0, 32)):
        cases = golden[key] if isinstance(golden[key], list) else [golden[key]]
        for c in cases:
            blk = np.frombuffer(bytes.fromhex(c["block"]), np.uint8)
            out = torch.zeros(n, device="cuda")
            kernels.dequant_rows(typ, dev(blk.copy()), 1, n, 0, 1, out)
            np.testing.assert_array_equal(host(out), np.array(c["want"], np.float32))


ATTN_SHAPES = [(6, 2, 64, 1), (6, 2, 64, 7), (6, 2, 64, 256), (6, 2, 64, 1000), (32, 8, 128, 1),
               (32, 8, 128, 300), (24, 8, 128, 33), (64, 8, 128, 4100), (32, 8, 128, 8193)]


@pytest.mark.parametrize("nh,nkv,hd,kv_len", ATTN_SHAPES)
def test_attn_decode(kernels, orc, nh, nkv, hd, kv_len):
    # backend/gpu/gpu_test.go:265 TestAttnDecode (+ long caches)
    rng = np.random.default_rng(7 + kv_len)
    q = randf(rng, nh * hd, 1)
    kc, vc = randf(rng, kv_len * nkv * hd, 1), randf(rng, kv_len * nkv * hd, 1)
    scale = np.float32(1 / math.sqrt(hd))
    want = orc.attn_decode(q, kc, vc, kv_len, nh, nkv, hd, float(scale))
    dout = torch.zeros(nh * hd, device="cuda")
    kernels.attn_decode(dev(q), dev(kc), dev(vc), dout, kv_len, nh, nkv, hd, float(scale))
    assert_close("AttnDecode", host(dout), want, 1e-5, 1e-4)
    # again: the split counters must have been reset
    kernels.attn_decode(dev(q), dev(kc), dev(vc), dout, kv_len, nh, nkv, hd, float(scale))
    assert_close("AttnDecode(again)", host(dout), want, 1e-5, 1e-4)


def test_argmax_device(kernels, orc):
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for x in (np.array([1, 3, 3, 2], np.float32), np.array([np.nan, 1, 2], np.float32),
              np.array([0, np.nan, 2], np.float32), np.random.default_rng(0).standard_normal(128256).astype(np.float32)):
        kernels.argmax(dev(x), x.size, out)
        assert int(host(out)[0]) == orc.argmax(x)


def test_ones(gb, kernels, cuda):
    # gpu.Ones, backend/gpu/gpu.go:157
    import ctypes as C

    p = C.c_void_p()
    gb._check(gb.lib().gb_gpu_ones(1000, C.byref(p)))
    out = torch.zeros(1000, device="cuda")
    zero = torch.zeros(1000, device="cuda")
    kernels.add(p.value, zero, out, 1000)
    assert host(out).tolist() == [1.0] * 1000
    gb._check(gb.lib().gb_free(p))


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)])
@pytest.mark.parametrize("typ", [Q4_0, Q4_K, Q6_K])
def test_gemv_sweep_shapes_vs_oracle(gb, orc, cuda, typ, rows, cols):
    # BASELINE config 2 at full size: the shapes and block recipe the bench's
    # GEMV sweep times (seed 0), against cpu.MatVecQ
    w = gb.synth_matrix(typ, rows, cols, seed=0)
    x = gb.synth_normal(0, 1, cols)
    want = orc.matvec_q(typ, w, x, rows, cols)
    lin = gb.Linear(typ, w, rows, cols)
    dy = torch.zeros(rows, device="cuda")
    for _ in range(2):
        lin.matvec(dev(x), dy)
    assert_close(f"sweep {typ} {rows}x{cols}", host(dy), want, 1e-4, 1e-4)
    lin.close()
