"""Generates the committed golden fixtures of tests/golden/.

* f16_known: the ten binary16 conversions of the reference's
  f16/f16_test.go:TestKnown (value -> expected half bits).
* q8_0 / q4_0: the known-answer blocks of quant/quant_test.go:TestQ8Q4
  (d = 0.5; Q8_0 quants j-16; Q4_0 nibbles lo=j, hi=15-j) with the values the
  reference test asserts.
* q4_k / q5_k / q6_k: blocks built here from chosen scales, mins and quants,
  packed by the ggml layout rules (6-bit scale/min packing of get_scale_min_k4;
  Q5_K fifth bits in qh; Q6_K ql/qh bit placement), with the expected values computed directly from the
  chosen numbers (d*sc*q - dmin*m and d*sc*(q-32)). All chosen values make the
  products exact in float32, so the expectations do not depend on rounding.
  The reference has no Q4_K/Q6_K/Q5_K known-answer test; these pin the decoders
  to the format, independently of the code under test.
* roundtrip.gguf: the file of gguf/gguf_test.go:TestRoundTrip (metadata and
  two tensors), written by the writer below, which follows gguf/writer.go.

Run: python tests/golden/make_golden.py (writes next to this file).
"""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def half_bits(x: float) -> int:
    return int(np.array([x], np.float16).view(np.uint16)[0])


def f16_known():
    # f16/f16_test.go:24-28
    cases = [(0.0, 0x0000), (1.0, 0x3C00), (-2.0, 0xC000), (65504.0, 0x7BFF), (1e-8, 0x0000),
             (5.960464e-8, 0x0001), (0.1, 0x2E66), (math.inf, 0x7C00), (1e5, 0x7C00),
             (3.14159, 0x4248)]
    return [{"x_bits": int(np.array([x], np.float32).view(np.uint32)[0]), "h": h} for x, h in cases]


def q8_0_block():
    # quant/quant_test.go:19-31
    blk = bytearray(34)
    blk[0:2] = struct.pack("<H", half_bits(0.5))
    for j in range(32):
        blk[2 + j] = (j - 16) & 0xFF
    return bytes(blk), [0.5 * (j - 16) for j in range(32)]


def q4_0_block():
    # quant/quant_test.go:33-45
    blk = bytearray(18)
    blk[0:2] = struct.pack("<H", half_bits(0.5))
    for j in range(16):
        blk[2 + j] = j | ((15 - j) << 4)
    want = [0.0] * 32
    for j in range(16):
        want[j] = 0.5 * (j - 8)
        want[j + 16] = 0.5 * (15 - j - 8)
    return bytes(blk), want


def pack_q4k_scales(sc, m):
    """Inverse of ggml get_scale_min_k4: 8 six-bit scales and mins -> 12 bytes."""
    s = [0] * 12
    for j in range(4):
        s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        s[j + 4] = (m[j] & 63) | ((m[j + 4] >> 4) << 6)
        s[j + 8] = (sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4)
    return bytes(s)


def q4_k_block(d, dmin, sc, m, q):
    """q: 256 quants 0..15 in element order."""
    blk = bytearray(144)
    blk[0:2] = struct.pack("<H", half_bits(d))
    blk[2:4] = struct.pack("<H", half_bits(dmin))
    blk[4:16] = pack_q4k_scales(sc, m)
    for chunk in range(4):
        for l in range(32):
            lo, hi = q[chunk * 64 + l], q[chunk * 64 + 32 + l]
            blk[16 + chunk * 32 + l] = lo | (hi << 4)
    want = []
    for e in range(256):
        j = e // 32
        want.append(d * sc[j] * q[e] - dmin * m[j])
    return bytes(blk), want


def q5_k_block(d, dmin, sc, m, q):
    """q: 256 five-bit quants 0..31 in element order. The published ggml
    block_q5_K layout: d, dmin, the Q4_K scale packing, qh[32] (bit 2j of byte
    l = fifth bit of element 64j+l, bit 2j+1 that of 64j+32+l), qs[128]."""
    blk = bytearray(176)
    blk[0:2] = struct.pack("<H", half_bits(d))
    blk[2:4] = struct.pack("<H", half_bits(dmin))
    blk[4:16] = pack_q4k_scales(sc, m)
    for chunk in range(4):
        for l in range(32):
            lo, hi = q[chunk * 64 + l], q[chunk * 64 + 32 + l]
            blk[48 + chunk * 32 + l] = (lo & 0xF) | ((hi & 0xF) << 4)
            blk[16 + l] |= ((lo >> 4) << (2 * chunk)) | ((hi >> 4) << (2 * chunk + 1))
    want = []
    for e in range(256):
        j = e // 32
        want.append(d * sc[j] * q[e] - dmin * m[j])
    return bytes(blk), want


def q6_k_block(d, scales, q):
    """scales: 16 int8; q: 256 six-bit quants 0..63 in element order."""
    ql, qh = bytearray(128), bytearray(64)
    for e in range(256):
        c, w = divmod(e, 128)
        quarter, l = divmod(w, 32)
        qv = q[e]
        bi = c * 64 + l + (quarter & 1) * 32
        if quarter >> 1:
            ql[bi] |= (qv & 0xF) << 4
        else:
            ql[bi] |= qv & 0xF
        qh[c * 32 + l] |= ((qv >> 4) & 3) << (2 * quarter)
    blk = bytes(ql) + bytes(qh) + bytes(s & 0xFF for s in scales) + struct.pack("<H", half_bits(d))
    want = []
    for e in range(256):
        c, w = divmod(e, 128)
        quarter, l = divmod(w, 32)
        is_ = l // 16
        sc = scales[c * 8 + is_ + 2 * quarter]
        want.append(d * sc * (q[e] - 32))
    return blk, want


# ---- a GGUF writer following gguf/writer.go ------------------------------------
def _s(b: bytearray, s: str):
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def _val(b: bytearray, t: int, v):
    fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q",
           11: "<q", 12: "<d"}
    if t == 8:
        _s(b, v)
    elif t == 9:
        et, items = v
        b += struct.pack("<IQ", et, len(items))
        for it in items:
            _val(b, et, it)
    else:
        b += struct.pack(fmt[t], v)


def write_gguf(kvs, tensors, alignment=32) -> bytes:
    """kvs: [(key, type, value)]; tensors: [(name, shape row-major, ggml type, bytes)]."""
    b = bytearray()
    b += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kvs))
    for k, t, v in kvs:
        _s(b, k)
        b += struct.pack("<I", t)
        _val(b, t, v)
    off = 0
    for name, shape, typ, data in tensors:
        _s(b, name)
        b += struct.pack("<I", len(shape))
        for d in reversed(shape):
            b += struct.pack("<Q", d)
        b += struct.pack("<IQ", typ, off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    while len(b) % alignment:
        b.append(0)
    for _, _, _, data in tensors:
        b += data
        while len(b) % alignment:
            b.append(0)
    return bytes(b)


def roundtrip_gguf() -> bytes:
    # gguf/gguf_test.go:11-37
    kvs = [("general.architecture", 8, "llama"), ("llama.block_count", 4, 2),
           ("llama.rope.freq_base", 6, 10000.0),
           ("tokenizer.ggml.tokens", 9, (8, ["<s>", "</s>", "hello"])),
           ("tokenizer.ggml.scores", 9, (6, [0.0, -1.0, 2.5])), ("x.flag", 7, True),
           ("x.big", 11, -7)]
    a = b"".join(struct.pack("<f", float(i)) for i in range(12))
    q = bytes(i & 0xFF for i in range(34 * 2 * 2))
    return write_gguf(kvs, [("a.weight", [4, 3], 0, a), ("q.weight", [2, 64], 8, q)])


def corrupt_base_gguf() -> bytes:
    # gguf/gguf_test.go:100-105
    return write_gguf([("k", 8, "v")], [("t", [8], 0, bytes(32))])


def main():
    rng = np.random.default_rng(20261201)
    out = {"f16_known": f16_known()}
    blk, want = q8_0_block()
    out["q8_0"] = {"block": blk.hex(), "want": want}
    blk, want = q4_0_block()
    out["q4_0"] = {"block": blk.hex(), "want": want}
    q4k = []
    # scales/mins with high bits set (j >= 4 use the packed upper bits), every
    # nibble value, and a second block with the extremes
    sc = [1, 2, 63, 17, 37, 48, 16, 63]
    m = [0, 5, 63, 31, 33, 20, 63, 1]
    qv = [int(x) for x in rng.integers(0, 16, 256)]
    qv[:16] = list(range(16))
    q4k.append((0.5, 0.25, sc, m, qv))
    q4k.append((2.0, 0.125, [63] * 8, [63, 0, 63, 0, 63, 0, 63, 0], [15 if i % 2 else 0 for i in range(256)]))
    out["q4_k"] = []
    for d, dmin, sc, m, qv in q4k:
        blk, want = q4_k_block(d, dmin, sc, m, qv)
        out["q4_k"].append({"block": blk.hex(), "want": want})
    q6k = []
    scales = [-32, -7, 1, 31, 5, -1, 12, -20, 30, 2, -3, 7, -16, 16, 9, -9]
    qv = [int(x) for x in rng.integers(0, 64, 256)]
    qv[:64] = list(range(64))
    q6k.append((0.25, scales, qv))
    q6k.append((1.0, [31] * 8 + [-32] * 8, [63 if i % 3 else 0 for i in range(256)]))
    out["q6_k"] = []
    for d, scales, qv in q6k:
        blk, want = q6_k_block(d, scales, qv)
        out["q6_k"].append({"block": blk.hex(), "want": want})
    # Q5_K (the reference lists the type but has no decoder): every 5-bit value,
    # high scale bits, and a block of extremes
    q5k = []
    qv = [int(x) for x in rng.integers(0, 32, 256)]
    qv[:32] = list(range(32))
    q5k.append((0.25, 0.5, [3, 63, 17, 1, 40, 33, 63, 16], [63, 2, 0, 31, 17, 48, 1, 63], qv))
    q5k.append((1.0, 0.0625, [63] * 8, [0, 63] * 4, [31 if i % 3 else 16 for i in range(256)]))
    out["q5_k"] = []
    for d, dmin, sc, m, qv in q5k:
        blk, want = q5_k_block(d, dmin, sc, m, qv)
        out["q5_k"].append({"block": blk.hex(), "want": want})
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    with open(os.path.join(HERE, "roundtrip.gguf"), "wb") as f:
        f.write(roundtrip_gguf())
    with open(os.path.join(HERE, "corrupt_base.gguf"), "wb") as f:
        f.write(corrupt_base_gguf())


if __name__ == "__main__":
    main()
