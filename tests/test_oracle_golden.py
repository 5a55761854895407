"""Pins the CPU oracle (oracle/oracle.c) to the reference's own known answers
(f16/f16_test.go, quant/quant_test.go) and to hand-derived Q4_K / Q6_K blocks,
and cross-checks its decoders against an independent numpy restatement."""
import math
import struct

import numpy as np
import pytest

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F32, F16, BF16 = 2, 8, 12, 13, 14, 0, 1, 30


def test_f16_known(orc, golden):
    # f16/f16_test.go:TestKnown
    for c in golden["f16_known"]:
        x = struct.unpack("<f", struct.pack("<I", c["x_bits"]))[0]
        assert orc.f16_from(x) == c["h"], (x, hex(c["h"]))
    assert math.isnan(orc.f16_to_f32(orc.f16_from(float("nan"))))


def test_f16_roundtrip_exhaustive(orc):
    # f16/f16_test.go:TestRoundTrip: every non-NaN half survives half->f32->half
    for h in range(1 << 16):
        if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
            continue
        assert orc.f16_from(orc.f16_to_f32(h)) == h, hex(h)


def test_f16_matches_numpy_rne(orc):
    # independent check of round-to-nearest-even on random float32 values
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 500)]).astype(np.float32)
    want = xs.astype(np.float16).view(np.uint16)
    for x, w in zip(xs, want):
        assert orc.f16_from(float(x)) == int(w)


def test_q8_q4_known_answers(orc, golden):
    # quant/quant_test.go:TestQ8Q4
    for key, typ in (("q8_0", Q8_0), ("q4_0", Q4_0)):
        blk = np.frombuffer(bytes.fromhex(golden[key]["block"]), np.uint8)
        got = orc.dequantize(typ, blk, 32)
        assert got.tolist() == golden[key]["want"]


@pytest.mark.parametrize("key,typ", [("q4_k", Q4_K), ("q5_k", Q5_K), ("q6_k", Q6_K)])
def test_kquant_hand_derived(orc, golden, key, typ):
    for case in golden[key]:
        blk = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
        got = orc.dequantize(typ, blk, 256)
        np.testing.assert_array_equal(got, np.array(case["want"], np.float32))


def test_dequantize_errors(orc):
    blk = np.zeros(144, np.uint8)
    with pytest.raises(ValueError):
        orc.dequantize(Q4_K, blk, 100)  # not a block multiple
    with pytest.raises(ValueError):
        orc.dequantize(Q4_K, blk[:100], 256)  # short data
    with pytest.raises(ValueError):
        orc.dequantize(99, blk, 32)  # unsupported


# ---- an independent numpy decoder (vectorised, float32 op by op) -----------
def np_half(b):
    return b.view(np.float16).astype(np.float32)


def np_dequant(typ, raw, n):
    raw = np.asarray(raw, np.uint8)
    if typ == Q4_0:
        blk = raw.reshape(-1, 18)
        d = np_half(blk[:, 0:2].copy())
        q = blk[:, 2:]
        lo = (q & 0xF).astype(np.float32) - np.float32(8)
        hi = (q >> 4).astype(np.float32) - np.float32(8)
        return np.concatenate([d * lo, d * hi], axis=1).reshape(-1)
    if typ == Q4_K:
        blk = raw.reshape(-1, 144)
        d, dmin = np_half(blk[:, 0:2].copy()), np_half(blk[:, 2:4].copy())
        s = blk[:, 4:16].astype(np.int32)
        sc = np.zeros((blk.shape[0], 8), np.int32)
        m = np.zeros((blk.shape[0], 8), np.int32)
        sc[:, :4] = s[:, :4] & 63
        m[:, :4] = s[:, 4:8] & 63
        sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
        m[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
        q = blk[:, 16:].reshape(-1, 4, 32)
        out = np.zeros((blk.shape[0], 256), np.float32)
        for c in range(4):
            for half, nib in ((0, q[:, c] & 0xF), (1, q[:, c] >> 4)):
                j = 2 * c + half
                dj = d[:, 0:1] * sc[:, j:j + 1].astype(np.float32)
                mj = dmin[:, 0:1] * m[:, j:j + 1].astype(np.float32)
                out[:, c * 64 + half * 32: c * 64 + half * 32 + 32] = dj * nib.astype(np.float32) - mj
        return out.reshape(-1)
    if typ == Q5_K:
        blk = raw.reshape(-1, 176)
        d, dmin = np_half(blk[:, 0:2].copy()), np_half(blk[:, 2:4].copy())
        s = blk[:, 4:16].astype(np.int32)
        sc = np.zeros((blk.shape[0], 8), np.int32)
        m = np.zeros((blk.shape[0], 8), np.int32)
        sc[:, :4] = s[:, :4] & 63
        m[:, :4] = s[:, 4:8] & 63
        sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
        m[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
        qh = blk[:, 16:48].astype(np.int32)
        q = blk[:, 48:].reshape(-1, 4, 32).astype(np.int32)
        out = np.zeros((blk.shape[0], 256), np.float32)
        for c in range(4):
            for half, nib in ((0, q[:, c] & 0xF), (1, q[:, c] >> 4)):
                j = 2 * c + half
                q5 = nib | (((qh >> j) & 1) << 4)
                dj = d[:, 0:1] * sc[:, j:j + 1].astype(np.float32)
                mj = dmin[:, 0:1] * m[:, j:j + 1].astype(np.float32)
                out[:, c * 64 + half * 32: c * 64 + half * 32 + 32] = dj * q5.astype(np.float32) - mj
        return out.reshape(-1)
    if typ == Q6_K:
        blk = raw.reshape(-1, 210)
        ql, qh, sc = blk[:, :128], blk[:, 128:192], blk[:, 192:208].view(np.int8)
        d = np_half(blk[:, 208:210].copy())
        out = np.zeros((blk.shape[0], 256), np.float32)
        for c in range(2):
            l0, h0, s0 = ql[:, c * 64:], qh[:, c * 32:], sc[:, c * 8:]
            for quarter in range(4):
                base = l0[:, (quarter & 1) * 32:(quarter & 1) * 32 + 32]
                nib = (base >> 4) if quarter >> 1 else (base & 0xF)
                q = (nib | (((h0[:, :32] >> (2 * quarter)) & 3) << 4)).astype(np.int32) - 32
                for is_ in range(2):
                    scv = s0[:, is_ + 2 * quarter].astype(np.float32)[:, None]
                    seg = slice(c * 128 + quarter * 32 + 16 * is_, c * 128 + quarter * 32 + 16 * is_ + 16)
                    out[:, seg] = (d * scv) * q[:, 16 * is_:16 * is_ + 16].astype(np.float32)
        return out.reshape(-1)
    raise ValueError(typ)


@pytest.mark.parametrize("typ,bs,ts", [(Q4_0, 32, 18), (Q4_K, 256, 144), (Q5_K, 256, 176), (Q6_K, 256, 210)])
def test_oracle_vs_independent_numpy(orc, typ, bs, ts):
    rng = np.random.default_rng(typ)
    nblk = 64
    raw = rng.integers(0, 256, nblk * ts, dtype=np.uint8)
    # finite binary16 scales (random bytes may encode inf/NaN)
    for b in range(nblk):
        for off in ((0,) if typ == Q4_0 else (0, 2) if typ in (Q4_K, Q5_K) else (208,)):
            raw[b * ts + off: b * ts + off + 2] = np.array([rng.normal(0, 0.01)], np.float16).view(np.uint8)
    got = orc.dequantize(typ, raw, nblk * bs)
    want = np_dequant(typ, raw, nblk * bs)
    np.testing.assert_array_equal(got, want)


def test_matvec_threads_bit_identical(orc, gb):
    raw = gb.synth_matrix(Q4_K, 96, 512, seed=3)
    x = gb.synth_normal(1, 2, 512)
    y1 = orc.matvec_q(Q4_K, raw, x, 96, 512, threads=1)
    y8 = orc.matvec_q(Q4_K, raw, x, 96, 512, threads=8)
    assert y1.tobytes() == y8.tobytes()


def test_softmax_and_argmax_rules(orc):
    x = np.array([1.0, 3.0, 3.0, -1.0], np.float32)
    s = orc.softmax(x, 1, 4)
    assert abs(float(s.sum()) - 1) < 1e-6
    assert orc.argmax(x) == 1  # first maximum wins
    assert orc.argmax(np.array([np.nan, 5, 6], np.float32)) == 0  # NaN at 0 is never beaten
    assert orc.argmax(np.array([1, np.nan, 6], np.float32)) == 2  # NaN never wins


def test_rope_vs_float64_numpy(orc):
    rng = np.random.default_rng(4)
    rows, nh, hd = 3, 2, 64
    x = rng.uniform(-2, 2, rows * nh * hd).astype(np.float32)
    pos = np.array([0, 7, 4095], np.int32)
    got = orc.rope(x, pos, None, rows, nh, hd, 10000.0)
    want = x.astype(np.float64).reshape(rows, nh, hd // 2, 2).copy()
    j = np.arange(hd // 2)
    for r in range(rows):
        th = pos[r] * np.power(10000.0, -2.0 * j / hd)
        c, s = np.cos(th), np.sin(th)
        x0, x1 = want[r, :, :, 0].copy(), want[r, :, :, 1].copy()
        want[r, :, :, 0] = x0 * c - x1 * s
        want[r, :, :, 1] = x0 * s + x1 * c
    np.testing.assert_allclose(got, want.reshape(-1).astype(np.float32), rtol=0, atol=2e-6)
