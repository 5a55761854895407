"""ctypes binding of oracle/liboracle.so, the CPU restatement of the reference's
pure-Go path (backend/cpu, quant, f16, gguf, cpuForward). Test infrastructure:
the checker the GPU path is compared against, never part of the product."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")

P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
_SIGS = {
    "or_block_size": (I, [I]), "or_type_size": (I, [I]), "or_row_bytes": (I64, [I, I64]),
    "or_f16_from": (C.c_uint16, [F]), "or_f16_to_f32": (F, [C.c_uint16]),
    "or_dequantize": (I, [I, P, I64, P, I64]), "or_row": (I, [I, P, I64, I, I64, P]),
    "or_rmsnorm": (None, [P, P, P, I, I, F]), "or_softmax": (None, [P, P, I, I]),
    "or_silu_mul": (None, [P, P, P, I64]), "or_add": (None, [P, P, P, I64]),
    "or_rope": (None, [P, P, P, I, I, I, F]), "or_matvec_f16": (None, [P, P, P, I, I, I]),
    "or_matvec_f32": (None, [P, P, P, I, I, I]), "or_matvec_q": (I, [I, P, I64, P, P, I, I, I, I]),
    "or_attn_decode": (None, [P, P, P, P, I, I, I, I, F]), "or_argmax": (C.c_int32, [P, I64]),
    "or_gguf_parse": (P, [P, C.c_size_t, C.c_char_p, I]), "or_gguf_free": (None, [P]),
    "or_gguf_version": (C.c_uint32, [P]), "or_gguf_alignment": (C.c_uint32, [P]),
    "or_gguf_n_tensors": (I, [P]), "or_gguf_n_kv": (I, [P]),
    "or_gguf_uint": (C.c_uint64, [P, C.c_char_p, C.c_uint64]),
    "or_gguf_float": (C.c_double, [P, C.c_char_p, C.c_double]),
    "or_gguf_string": (None, [P, C.c_char_p, C.c_char_p, C.c_char_p, I]),
    "or_gguf_tensor": (I, [P, C.c_char_p, C.POINTER(I), C.POINTER(I), P, C.POINTER(P), C.POINTER(C.c_uint64)]),
    "or_model_open": (P, [P, C.c_size_t, I, I, C.c_char_p, I]), "or_model_free": (None, [P]),
    "or_model_forward": (I, [P, C.c_int32, I, P, I]), "or_model_set_kv": (I, [P, I, I, I, P, P]),
    "or_model_kcache": (P, [P, I]), "or_model_vcache": (P, [P, I]),
    "or_exp_nonpos": (F, [F]), "or_uniform24": (F, [C.c_uint64, C.c_uint64]),
    "or_sample": (C.c_int32, [P, I, P, P, I, C.c_uint64]),
    "or_synth_preset": (I, [I, P]), "or_synth_model": (I, [P, C.POINTER(P), C.POINTER(C.c_size_t)]),
    "or_synth_free": (None, [P]), "or_synth_kv_normal": (I, [C.c_uint64, I, I, I, I, I, P, P]),
}


class SampleParams(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int), ("reserved", C.c_int),
                ("seed", C.c_uint64)]

class SynthSpec(C.Structure):
    """or_synth_spec: the shape, weight mix and seed of a synthetic model."""
    _fields_ = [("layers", C.c_int), ("dim", C.c_int), ("ffn", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("ctx_len", C.c_int),
                ("rope_base", C.c_float), ("eps", C.c_float), ("mix", C.c_int), ("seed", C.c_uint64)]


_lib = None


def build() -> None:
    """Compile the restatement (make -C oracle)."""
    subprocess.run(["make", "-C", ORACLE_DIR, "-s", "CC=" + _cc()], check=True)


def _cc() -> str:
    # a gcc whose toolchain has libm/libpthread; prefer the system one
    return "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        l = C.CDLL(ORACLE_SO)
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = res, args
        _lib = l
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def f16_from(x: float) -> int:
    return int(lib().or_f16_from(x))


def f16_to_f32(h: int) -> float:
    return float(lib().or_f16_to_f32(h))


def dequantize(typ: int, data: np.ndarray, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data, np.uint8)
    out = np.empty(n, np.float32)
    rc = lib().or_dequantize(typ, _p(data), data.nbytes, _p(out), n)
    if rc:
        raise ValueError(f"or_dequantize: {rc}")
    return out


def rmsnorm(x, w, rows, n, eps):
    out = np.empty_like(x)
    lib().or_rmsnorm(_p(x), _p(w), _p(out), rows, n, eps)
    return out


def softmax(x, rows, n):
    out = np.empty_like(x)
    lib().or_softmax(_p(x), _p(out), rows, n)
    return out


def silu_mul(g, u):
    out = np.empty_like(g)
    lib().or_silu_mul(_p(g), _p(u), _p(out), g.size)
    return out


def add(a, b):
    out = np.empty_like(a)
    lib().or_add(_p(a), _p(b), _p(out), a.size)
    return out


def rope(x, pos, freq, rows, n_heads, head_dim, base):
    y = np.array(x, np.float32, copy=True)
    pos = np.ascontiguousarray(pos, np.int32)
    lib().or_rope(_p(y), _p(pos), _p(freq) if freq is not None else None, rows, n_heads, head_dim, base)
    return y


def matvec_f16(w16, x, rows, cols, batch):
    y = np.empty(batch * rows, np.float32)
    lib().or_matvec_f16(_p(w16), _p(x), _p(y), rows, cols, batch)
    return y


def matvec_f32(w, x, rows, cols, batch):
    y = np.empty(batch * rows, np.float32)
    lib().or_matvec_f32(_p(w), _p(x), _p(y), rows, cols, batch)
    return y


def matvec_q(typ, w, x, rows, cols, batch=1, threads=None):
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(batch * rows, np.float32)
    rc = lib().or_matvec_q(typ, _p(w), w.nbytes, _p(x), _p(y), rows, cols, batch, threads or os.cpu_count())
    if rc:
        raise ValueError(f"or_matvec_q: {rc}")
    return y


def attn_decode(q, kc, vc, kv_len, n_heads, n_kv, head_dim, scale):
    out = np.empty(n_heads * head_dim, np.float32)
    lib().or_attn_decode(_p(q), _p(kc), _p(vc), _p(out), kv_len, n_heads, n_kv, head_dim, scale)
    return out


def argmax(x) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().or_argmax(_p(x), x.size))


def sample(logits, temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64, seed=0,
           recent=(), counter=0) -> int:
    """The sampler's rule on the host (the checker of gb_gpu_sample)."""
    x = np.ascontiguousarray(logits, np.float32)
    r = np.ascontiguousarray(np.asarray(recent, np.int32))
    prm = SampleParams(temperature, top_k, top_p, repeat_penalty, repeat_last_n, 0, seed)
    return int(lib().or_sample(_p(x), x.size, C.byref(prm), _p(r) if r.size else None, r.size, counter))


def exp_nonpos(x: float) -> float:
    return float(lib().or_exp_nonpos(x))


def uniform24(seed: int, counter: int) -> float:
    return float(lib().or_uniform24(seed, counter))


class Gguf:
    def __init__(self, data: bytes):
        self._buf = C.create_string_buffer(data, len(data)) if data else C.create_string_buffer(1)
        err = C.create_string_buffer(256)
        self.h = lib().or_gguf_parse(C.addressof(self._buf), len(data), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())

    def close(self):
        if self.h:
            lib().or_gguf_free(self.h)
            self.h = None


class OracleModel:
    """cpuForward (model/model_test.go:114) over a GGUF image."""

    def __init__(self, image: np.ndarray, max_len: int, kv_f16: bool):
        self.image = np.ascontiguousarray(image, np.uint8)
        err = C.create_string_buffer(256)
        self.h = lib().or_model_open(_p(self.image), self.image.nbytes, max_len, int(kv_f16), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())

    def forward(self, token: int, pos: int, vocab: int, threads: int | None = None) -> np.ndarray:
        out = np.empty(vocab, np.float32)
        rc = lib().or_model_forward(self.h, token, pos, _p(out), threads or os.cpu_count())
        if rc:
            raise ValueError(f"or_model_forward: {rc}")
        return out

    def set_kv(self, layer, pos0, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        rc = lib().or_model_set_kv(self.h, layer, pos0, k.shape[0], _p(k), _p(v))
        if rc:
            raise ValueError("or_model_set_kv")

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None


def synth_preset(preset: int, **over) -> SynthSpec:
    s = SynthSpec()
    if lib().or_synth_preset(preset, C.byref(s)):
        raise ValueError(f"unknown preset {preset}")
    for k, v in over.items():
        setattr(s, k, v)
    return s


def synth_spec(**kw) -> SynthSpec:
    """Defaults as the product's synth_spec: vocab 128256, ctx 2048, Q4_K_M, seed 0."""
    s = SynthSpec(vocab=128256, rope_base=500000.0, eps=1e-5, ctx_len=2048, mix=1, seed=0)
    for k, v in kw.items():
        setattr(s, k, v)
    if "head_dim" not in kw:
        s.head_dim = s.dim // s.heads
    return s


def synth_model(spec: SynthSpec) -> np.ndarray:
    """The synthetic GGUF image of spec (the bytes the product's generator writes)."""
    p, n = C.c_void_p(), C.c_size_t()
    if lib().or_synth_model(C.byref(spec), C.byref(p), C.byref(n)):
        raise ValueError("or_synth_model failed")
    try:
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), (n.value,)).copy()
    finally:
        lib().or_synth_free(p)


def synth_kv_normal(seed: int, layer: int, pos0: int, n: int, kv_dim: int, f16: bool):
    k = np.empty((n, kv_dim), np.float32)
    v = np.empty((n, kv_dim), np.float32)
    if lib().or_synth_kv_normal(seed, layer, pos0, n, kv_dim, int(f16), _p(k), _p(v)):
        raise ValueError("or_synth_kv_normal failed")
    return k, v
