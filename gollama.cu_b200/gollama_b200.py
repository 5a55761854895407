"""Python mirror of the gollama-b200 C ABI (include/gollama_b200.h) over ctypes.

The classes follow the reference's Go API for the decode path:
``Kernels`` is backend/gpu's *Kernels (backend/gpu/gpu.go:28-167), ``Linear``
is model.Linear (model/model.go:67-118), ``Model`` is model.Model
(model/model.go:134-392) and ``argmax`` is model.Argmax (model/model.go:376).
Errors surface as ``GollamaError`` carrying the library's status code and its
message, worded like the reference's Go errors.

Device buffers are passed as integers (device addresses) or as any object
with ``data_ptr()`` (e.g. torch tensors); this module itself needs neither
torch nor a GPU to import, so it loads on CPU-only machines.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgollama_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "gollama_b200.h")

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_IO, ERR_NCCL, ERR_TIMEOUT, ERR_DEVICE = range(8)
F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 30
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144),
         Q5_K: (256, 176), Q6_K: (256, 210)}


def row_bytes(typ: int, n: int) -> int:
    """gguf/types.go:81 RowBytes."""
    bs, ts = BLOCK[typ]
    return n // bs * ts


class GollamaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "dim", "ffn", "heads", "kv_heads", "head_dim",
                                        "vocab", "ctx_len")] + \
               [("rope_base", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int) for n in ("max_len", "kv_f16", "tp_rank", "tp_world")]


class ModelOpts(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("device", "max_len", "kv_f16", "use_graph", "tp_rank",
                                        "tp_world")] + [("nccl_id", C.c_void_p)]


class SynthSpec(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "dim", "ffn", "heads", "kv_heads", "head_dim",
                                        "vocab", "ctx_len")] + \
               [("rope_base", C.c_float), ("eps", C.c_float), ("mix", C.c_int),
                ("seed", C.c_uint64)]


class SampleParams(C.Structure):
    """gb_sample_params: the on-device sampler's rule (include/gollama_b200.h)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int), ("reserved", C.c_int),
                ("seed", C.c_uint64)]


def sample_params(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64,
                  seed=0) -> SampleParams:
    return SampleParams(temperature, top_k, top_p, repeat_penalty, repeat_last_n, 0, seed)


_lib = None
P, I, U64, F, D, S = C.c_void_p, C.c_int, C.c_uint64, C.c_float, C.c_double, C.c_size_t
_SIGS = {
    "gb_last_error": (C.c_char_p, []), "gb_version": (C.c_char_p, []),
    "gb_gpu_load": (I, [I, C.POINTER(P)]), "gb_gpu_len": (I, [P]), "gb_gpu_close": (I, [P]),
    "gb_gpu_rmsnorm": (I, [P, P, P, P, P, I, I, F]), "gb_gpu_softmax": (I, [P, P, P, P, I, I]),
    "gb_gpu_silu_mul": (I, [P, P, P, P, P, I]), "gb_gpu_add": (I, [P, P, P, P, P, I]),
    "gb_gpu_rope": (I, [P, P, P, P, P, I, I, I, F]),
    "gb_gpu_attn_decode": (I, [P, P, P, P, P, P, I, I, I, I, F]),
    "gb_gpu_attn_decode_noalloc": (I, [P, P, P, P, P, P, I, I, I, I, F]),
    "gb_gpu_matvec_f16": (I, [P, P, P, P, P, I, I, I]), "gb_gpu_matvec_f32": (I, [P, P, P, P, P, I, I, I]),
    "gb_gpu_matvec_q": (I, [P, P, I, P, P, P, I, I, I]), "gb_gpu_ones": (I, [I, C.POINTER(P)]),
    "gb_free": (I, [P]), "gb_gpu_dequant_rows": (I, [P, P, I, P, I, I, I, I, P]),
    "gb_gpu_argmax": (I, [P, P, P, I, P]),
    "gb_gpu_peer_resid": (I, [P, P, I, P, P, P, I, I, P, I, P, C.c_uint, P]),
    "gb_gpu_peer_resid_tagged": (I, [P, P, I, P, P, I, I, P, I, P, C.c_uint, P]), "gb_gpu_sample": (I, [P, P, P, I, P, P, I, U64, P]),
    "gb_gpu_attn_decode_paged": (I, [P, P, P, P, P, I, P, P, I, I, I, I, I, I, I, F, P]),
    "gb_model_set_sampler": (I, [P, P]), "gb_model_prefill": (I, [P, P, I, I, P]),
    "gb_model_cache_f16_weights": (I, [P, C.POINTER(S)]),
    "gb_linear_matmul_f16": (I, [P, P, P, I, P]), "gb_linear_cache_f16_weights": (I, [P, C.POINTER(S)]),
    "gb_engine_create": (I, [P, I, I, I, C.POINTER(P)]), "gb_engine_add": (I, [P, C.POINTER(I)]),
    "gb_engine_release": (I, [P, I]), "gb_engine_seq_len": (I, [P, I]), "gb_engine_free_pages": (I, [P]),
    "gb_engine_step": (I, [P, I, P, P, P, P]), "gb_engine_free": (I, [P]),
    "gb_linear_upload": (I, [I, I, P, S, I, I, C.POINTER(P)]), "gb_linear_matvec": (I, [P, P, P, P]),
    "gb_linear_info": (I, [P, C.POINTER(I), C.POINTER(I), C.POINTER(I), C.POINTER(S)]),
    "gb_linear_free": (I, [P]),
    "gb_model_opts_default": (None, [P]), "gb_model_load": (I, [C.c_char_p, P, C.POINTER(P)]),
    "gb_model_load_mem": (I, [P, S, P, C.POINTER(P)]), "gb_model_config": (I, [P, P]),
    "gb_model_forward": (I, [P, C.c_int32, I, P]), "gb_model_next": (I, [P, C.c_int32, I, P]),
    "gb_model_generate": (I, [P, C.c_int32, I, I, P]), "gb_model_fill_kv_normal": (I, [P, U64, I]),
    "gb_model_start": (I, [P, C.c_int32, I]), "gb_model_decode_async": (I, [P, I]),
    "gb_model_read_tokens": (I, [P, I, I, P]),
    "gb_model_read_kv": (I, [P, I, I, I, P, P]), "gb_model_stream": (P, [P]),
    "gb_model_profile_step": (I, [P, C.c_int32, I, P, P]),
    "gb_model_step_bytes": (I, [P, I, C.POINTER(D), C.POINTER(D)]),
    "gb_model_launches_per_step": (I, [P]), "gb_model_close": (I, [P]),
    "gb_argmax": (C.c_int32, [P, C.c_int64]),
    "gb_gguf_parse": (I, [P, S, C.POINTER(P)]), "gb_gguf_open": (I, [C.c_char_p, C.POINTER(P)]),
    "gb_gguf_close": (I, [P]),
    "gb_gguf_header": (I, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(I), C.POINTER(I)]),
    "gb_gguf_uint": (U64, [P, C.c_char_p, U64]), "gb_gguf_float": (D, [P, C.c_char_p, D]),
    "gb_gguf_string": (I, [P, C.c_char_p, C.c_char_p, P, I]),
    "gb_gguf_key": (C.c_char_p, [P, I, C.POINTER(I)]),
    "gb_gguf_array_len": (I, [P, C.c_char_p, C.POINTER(I)]),
    "gb_gguf_array_float": (D, [P, C.c_char_p, I]),
    "gb_gguf_array_string": (I, [P, C.c_char_p, I, P, I]),
    "gb_gguf_tensor": (I, [P, C.c_char_p, C.POINTER(I), C.POINTER(I), P, C.POINTER(U64),
                           C.POINTER(U64), C.POINTER(P)]),
    "gb_gguf_tensor_at": (C.c_char_p, [P, I]),
    "gb_tp_unique_id": (I, [P]),
    "gb_synth_preset": (I, [I, P]), "gb_synth_model": (I, [P, C.POINTER(P), C.POINTER(S)]),
    "gb_synth_model_file": (I, [P, C.c_char_p]), "gb_synth_free": (None, [P]),
    "gb_synth_matrix": (I, [I, I, I, U64, C.c_uint32, F, P]),
    "gb_synth_normal": (I, [U64, C.c_uint32, C.c_int64, P]),
    "gb_synth_kv_normal": (I, [U64, I, I, I, I, I, P, P]),
}


def lib() -> C.CDLL:
    """Load libgollama_b200.so (built in-tree by `make -C gollama.cu_b200`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GollamaError(ERR_IO, f"{LIB_PATH} is not built (run make -C gollama.cu_b200)")
        l = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def declared_functions() -> list[str]:
    """Every function include/gollama_b200.h declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gb_[a-z0-9_]+)\s*\(", src)))


def _check(rc: int) -> None:
    if rc != OK:
        raise GollamaError(rc, lib().gb_last_error().decode())


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot pass {type(x)} as a pointer")


def _stream(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


def argmax(logits: np.ndarray) -> int:
    """model.Argmax (model/model.go:376): the first maximum wins."""
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().gb_argmax(a.ctypes.data, a.size))


class Kernels:
    """backend/gpu's *Kernels: gpu.Load (backend/gpu/gpu.go:35) and the launch methods."""

    def __init__(self, device: int = 0):
        h = P()
        _check(lib().gb_gpu_load(device, C.byref(h)))
        self.h = h

    def __len__(self) -> int:
        return lib().gb_gpu_len(self.h)

    def close(self) -> None:
        if self.h:
            _check(lib().gb_gpu_close(self.h))
            self.h = None

    def rms_norm(self, x, w, out, rows, n, eps, stream=None):
        _check(lib().gb_gpu_rmsnorm(self.h, _stream(stream), _ptr(x), _ptr(w), _ptr(out), rows, n, eps))

    def softmax(self, x, out, rows, n, stream=None):
        _check(lib().gb_gpu_softmax(self.h, _stream(stream), _ptr(x), _ptr(out), rows, n))

    def silu_mul(self, gate, up, out, n, stream=None):
        _check(lib().gb_gpu_silu_mul(self.h, _stream(stream), _ptr(gate), _ptr(up), _ptr(out), n))

    def add(self, a, b, out, n, stream=None):
        _check(lib().gb_gpu_add(self.h, _stream(stream), _ptr(a), _ptr(b), _ptr(out), n))

    def rope(self, x, pos, freq, rows, n_heads, head_dim, base, stream=None):
        _check(lib().gb_gpu_rope(self.h, _stream(stream), _ptr(x), _ptr(pos), _ptr(freq), rows,
                                 n_heads, head_dim, base))

    def attn_decode(self, q, kc, vc, out, kv_len, n_heads, n_kv, head_dim, scale, stream=None):
        _check(lib().gb_gpu_attn_decode(self.h, _stream(stream), _ptr(q), _ptr(kc), _ptr(vc), _ptr(out),
                                        kv_len, n_heads, n_kv, head_dim, scale))

    def attn_decode_noalloc(self, q, kc, vc, out, kv_len, n_heads, n_kv, head_dim, scale, stream=None):
        """gb_gpu_attn_decode_noalloc: scratch in fixed device arrays (no allocation)."""
        _check(lib().gb_gpu_attn_decode_noalloc(self.h, _stream(stream), _ptr(q), _ptr(kc), _ptr(vc),
                                                _ptr(out), kv_len, n_heads, n_kv, head_dim, scale))

    def matvec_f16(self, w, x, y, rows, cols, batch, stream=None):
        _check(lib().gb_gpu_matvec_f16(self.h, _stream(stream), _ptr(w), _ptr(x), _ptr(y), rows, cols, batch))

    def matvec_f32(self, w, x, y, rows, cols, batch, stream=None):
        _check(lib().gb_gpu_matvec_f32(self.h, _stream(stream), _ptr(w), _ptr(x), _ptr(y), rows, cols, batch))

    def matvec_q(self, typ, w, x, y, rows, cols, batch, stream=None):
        _check(lib().gb_gpu_matvec_q(self.h, _stream(stream), typ, _ptr(w), _ptr(x), _ptr(y), rows, cols, batch))

    def dequant_rows(self, typ, w, rows, cols, row0, nrows, out, stream=None):
        _check(lib().gb_gpu_dequant_rows(self.h, _stream(stream), typ, _ptr(w), rows, cols, row0, nrows, _ptr(out)))

    def argmax(self, x, n, out, stream=None):
        _check(lib().gb_gpu_argmax(self.h, _stream(stream), _ptr(x), n, _ptr(out)))

    def peer_resid(self, world, bufs, flags, step, slot, dim, x, n, ssq, wait_limit=0, status=None, stream=None):
        """gb_gpu_peer_resid: x += the ranks' partials of `slot` once every flag shows *step + 1.
        bufs / flags: device arrays of `world` device pointers."""
        _check(lib().gb_gpu_peer_resid(self.h, _stream(stream), world, _ptr(bufs), _ptr(flags), _ptr(step), slot,
                                       dim, _ptr(x), n, _ptr(ssq), wait_limit, _ptr(status)))

    def peer_resid_tagged(self, world, bufs, step, slot, dim, x, n, ssq, wait_limit=0, status=None, stream=None):
        """gb_gpu_peer_resid_tagged: x += the ranks' partials of `slot` once every rank's word of an
        element carries the tag *step + 1. bufs: `world` device pointers (ints) to the ranks'
        [slots][dim] arrays of 64-bit tagged words."""
        arr = (C.c_uint64 * world)(*[int(b) for b in bufs])
        _check(lib().gb_gpu_peer_resid_tagged(self.h, _stream(stream), world, C.cast(arr, P), _ptr(step), slot,
                                              dim, _ptr(x), n, _ptr(ssq), wait_limit, _ptr(status)))

    def attn_decode_paged(self, q, k_pool, v_pool, kv_f16, block_table, seq_lens, batch, max_pages, n_pages,
                          page_size, n_heads, n_kv, head_dim, scale, out, stream=None):
        _check(lib().gb_gpu_attn_decode_paged(self.h, _stream(stream), _ptr(q), _ptr(k_pool), _ptr(v_pool),
                                              int(kv_f16), _ptr(block_table), _ptr(seq_lens), batch, max_pages,
                                              n_pages, page_size, n_heads, n_kv, head_dim, scale, _ptr(out)))

    def sample(self, logits, n, params: SampleParams, recent, n_recent, counter, out, stream=None):
        _check(lib().gb_gpu_sample(self.h, _stream(stream), _ptr(logits), n, C.byref(params),
                                   _ptr(recent) if n_recent else None, n_recent, counter, _ptr(out)))


class Linear:
    """model.Linear in the tiled layout: uploadLinear (model/model.go:77) + MatVec (:109)."""

    def __init__(self, typ: int, raw: np.ndarray, rows: int, cols: int, device: int = 0):
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        h = P()
        _check(lib().gb_linear_upload(device, typ, raw.ctypes.data, raw.nbytes, rows, cols, C.byref(h)))
        self.h, self.typ, self.rows, self.cols = h, typ, rows, cols

    def matvec(self, x, y, stream=None):
        _check(lib().gb_linear_matvec(self.h, _stream(stream), _ptr(x), _ptr(y)))

    def matmul_f16(self, x16, T: int, y, stream=None):
        """y[T][rows] = x16[T][cols] W^T on the tensor cores (x16 binary16, y float32)."""
        _check(lib().gb_linear_matmul_f16(self.h, _stream(stream), _ptr(x16), T, _ptr(y)))

    def cache_f16_weights(self) -> int:
        """Keep the binary16 copy of the weights for matmul_f16 (bit-identical
        results); its device bytes."""
        n = S(0)
        _check(lib().gb_linear_cache_f16_weights(self.h, C.byref(n)))
        return n.value

    def weight_bytes(self) -> int:
        s = S()
        _check(lib().gb_linear_info(self.h, None, None, None, C.byref(s)))
        return s.value

    def close(self):
        if self.h:
            _check(lib().gb_linear_free(self.h))
            self.h = None


def model_opts(**kw) -> ModelOpts:
    o = ModelOpts()
    lib().gb_model_opts_default(C.byref(o))
    nccl_id = kw.pop("nccl_id", None)
    for k, v in kw.items():
        setattr(o, k, int(v))
    if nccl_id is not None:
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        o._nccl_buf = buf  # keep alive
        o.nccl_id = C.addressof(buf)
    return o


class Model:
    """model.Model: Load (model/model.go:160), Forward (:313), Close (:387)."""

    def __init__(self, source, **opts):
        o = model_opts(**opts)
        h = P()
        if isinstance(source, (bytes, bytearray, memoryview)):
            buf = (C.c_char * len(source)).from_buffer_copy(source) if not isinstance(source, bytearray) \
                else (C.c_char * len(source)).from_buffer(source)
            _check(lib().gb_model_load_mem(C.addressof(buf), len(source), C.byref(o), C.byref(h)))
        elif isinstance(source, SynthImage):
            _check(lib().gb_model_load_mem(source.ptr, source.size, C.byref(o), C.byref(h)))
        else:
            _check(lib().gb_model_load(os.fsencode(source), C.byref(o), C.byref(h)))
        self.h = h
        c = Config()
        _check(lib().gb_model_config(h, C.byref(c)))
        self.config = c
        self._logits = np.empty(c.vocab, dtype=np.float32)

    def forward(self, token: int, pos: int, out: np.ndarray | None = None) -> np.ndarray:
        """Logits of token at pos; the returned array is reused by the next call (like the reference)."""
        dst = self._logits if out is None else out
        _check(lib().gb_model_forward(self.h, token, pos, dst.ctypes.data))
        return dst

    def forward_no_logits(self, token: int, pos: int) -> None:
        _check(lib().gb_model_forward(self.h, token, pos, None))

    def next(self, token: int, pos: int) -> int:
        n = C.c_int32()
        _check(lib().gb_model_next(self.h, token, pos, C.byref(n)))
        return n.value

    def generate(self, token: int, pos: int, n: int) -> np.ndarray:
        out = np.empty(max(n, 1), dtype=np.int32)
        _check(lib().gb_model_generate(self.h, token, pos, n, out.ctypes.data))
        return out[:n]

    def prefill(self, tokens, pos0: int = 0, out: np.ndarray | None = None) -> np.ndarray:
        """Feed tokens at pos0.. (batched); the logits of the last one."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        if out is None:
            out = self._logits
        _check(lib().gb_model_prefill(self.h, t.ctypes.data, t.size, pos0, out.ctypes.data))
        return out

    def cache_f16_weights(self) -> int:
        """Keep a binary16 copy of every weight matrix for prefill and the
        engine (bit-identical results); the device bytes it took."""
        n = S(0)
        _check(lib().gb_model_cache_f16_weights(self.h, C.byref(n)))
        return n.value

    def set_sampler(self, params: SampleParams | None) -> None:
        """Token rule of next/generate/decode_async: None = greedy argmax."""
        _check(lib().gb_model_set_sampler(self.h, C.byref(params) if params is not None else None))

    def start(self, token: int, pos: int) -> None:
        _check(lib().gb_model_start(self.h, token, pos))

    def decode_async(self, n: int) -> None:
        _check(lib().gb_model_decode_async(self.h, n))

    def read_tokens(self, pos0: int, n: int) -> np.ndarray:
        out = np.empty(max(n, 1), dtype=np.int32)
        _check(lib().gb_model_read_tokens(self.h, pos0, n, out.ctypes.data))
        return out[:n]

    def fill_kv_normal(self, seed: int, n_pos: int) -> None:
        _check(lib().gb_model_fill_kv_normal(self.h, seed, n_pos))

    def read_kv(self, layer: int, pos0: int, n: int):
        kvl = self.config.kv_heads * self.config.head_dim // self.config.tp_world
        k = np.empty((n, kvl), np.float32)
        v = np.empty((n, kvl), np.float32)
        _check(lib().gb_model_read_kv(self.h, layer, pos0, n, k.ctypes.data, v.ctypes.data))
        return k, v

    def stream(self) -> int:
        return lib().gb_model_stream(self.h) or 0

    def profile_step(self, token: int, pos: int):
        ms = np.zeros(7, np.float32)
        n = np.zeros(7, np.int32)
        _check(lib().gb_model_profile_step(self.h, token, pos, ms.ctypes.data, n.ctypes.data))
        names = ["qkv", "attention", "o_proj", "gate_up", "down", "lm_head", "other"]
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(names)}

    def step_bytes(self, kv_len: int):
        b, g = D(), D()
        _check(lib().gb_model_step_bytes(self.h, kv_len, C.byref(b), C.byref(g)))
        return b.value, g.value

    def launches_per_step(self) -> int:
        return lib().gb_model_launches_per_step(self.h)

    def close(self):
        if self.h:
            _check(lib().gb_model_close(self.h))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Engine:
    """Continuous batching over a Model: paged KV, one batched pass per step."""

    def __init__(self, model: "Model", page_size: int = 16, n_pages: int = 1024, max_batch: int = 64):
        h = P()
        _check(lib().gb_engine_create(model.h, page_size, n_pages, max_batch, C.byref(h)))
        self.h, self.model, self.vocab = h, model, model.config.vocab

    def add(self) -> int:
        i = C.c_int()
        _check(lib().gb_engine_add(self.h, C.byref(i)))
        return i.value

    def release(self, seq_id: int) -> None:
        _check(lib().gb_engine_release(self.h, seq_id))

    def seq_len(self, seq_id: int) -> int:
        return lib().gb_engine_seq_len(self.h, seq_id)

    def free_pages(self) -> int:
        return lib().gb_engine_free_pages(self.h)

    def step(self, seq_ids, tokens, logits: bool = True):
        """One row per (sequence, token); a sequence listed k times takes its next k
        positions in the order listed. Returns (logits [n][vocab] or None, next tokens [n])."""
        ids = np.ascontiguousarray(np.asarray(seq_ids, np.int32))
        toks = np.ascontiguousarray(np.asarray(tokens, np.int32))
        n = ids.size
        out = np.empty((n, self.vocab), np.float32) if logits else None
        nxt = np.empty(n, np.int32)
        _check(lib().gb_engine_step(self.h, n, ids.ctypes.data, toks.ctypes.data,
                                    out.ctypes.data if logits else None, nxt.ctypes.data))
        return out, nxt

    def close(self):
        if self.h:
            _check(lib().gb_engine_free(self.h))
            self.h = None


class SynthImage:
    """A synthetic GGUF image in host memory (gb_synth_model)."""

    def __init__(self, spec: SynthSpec):
        p, n = P(), S()
        _check(lib().gb_synth_model(C.byref(spec), C.byref(p), C.byref(n)))
        self.ptr, self.size, self.spec = p.value, n.value, spec

    def view(self) -> np.ndarray:
        return np.ctypeslib.as_array((C.c_uint8 * self.size).from_address(self.ptr))

    def close(self):
        if self.ptr:
            lib().gb_synth_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_preset(preset: int, **over) -> SynthSpec:
    s = SynthSpec()
    _check(lib().gb_synth_preset(preset, C.byref(s)))
    for k, v in over.items():
        setattr(s, k, v)
    return s


def synth_spec(**kw) -> SynthSpec:
    s = SynthSpec()
    s.vocab, s.rope_base, s.eps, s.ctx_len, s.mix, s.seed = 128256, 500000.0, 1e-5, 2048, 1, 0
    for k, v in kw.items():
        setattr(s, k, v)
    if "head_dim" not in kw:
        s.head_dim = s.dim // s.heads
    return s


def synth_matrix(typ: int, rows: int, cols: int, seed: int = 0, tensor_id: int = 0,
                 sigma: float = 0.0) -> np.ndarray:
    buf = np.empty(rows * row_bytes(typ, cols), dtype=np.uint8)
    _check(lib().gb_synth_matrix(typ, rows, cols, seed, tensor_id, sigma, buf.ctypes.data))
    return buf


def synth_normal(seed: int, stream_id: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(lib().gb_synth_normal(seed, stream_id, n, out.ctypes.data))
    return out


def synth_kv_normal(seed: int, layer: int, pos0: int, n: int, kv_dim: int, f16: bool):
    k = np.empty((n, kv_dim), np.float32)
    v = np.empty((n, kv_dim), np.float32)
    _check(lib().gb_synth_kv_normal(seed, layer, pos0, n, kv_dim, int(f16), k.ctypes.data, v.ctypes.data))
    return k, v


def tp_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(lib().gb_tp_unique_id(buf))
    return bytes(buf)


class Gguf:
    """gguf.File over the library's reader (gguf/gguf.go)."""

    def __init__(self, data: bytes | None = None, path: str | None = None):
        h = P()
        if path is not None:
            _check(lib().gb_gguf_open(os.fsencode(path), C.byref(h)))
            self._buf = None
        else:
            self._buf = C.create_string_buffer(bytes(data), len(data)) if data else C.create_string_buffer(1)
            _check(lib().gb_gguf_parse(C.addressof(self._buf), len(data or b""), C.byref(h)))
        self.h = h

    def header(self):
        v, a, nk, nt = C.c_uint32(), C.c_uint32(), I(), I()
        _check(lib().gb_gguf_header(self.h, C.byref(v), C.byref(a), C.byref(nk), C.byref(nt)))
        return v.value, a.value, nk.value, nt.value

    def uint(self, key, default=0):
        return lib().gb_gguf_uint(self.h, key.encode(), default)

    def float(self, key, default=0.0):
        return lib().gb_gguf_float(self.h, key.encode(), default)

    def string(self, key, default=""):
        buf = C.create_string_buffer(4096)
        _check(lib().gb_gguf_string(self.h, key.encode(), default.encode(), buf, 4096))
        return buf.value.decode()

    def keys(self):
        out, i, t = [], 0, I()
        while True:
            k = lib().gb_gguf_key(self.h, i, C.byref(t))
            if k is None:
                return out
            out.append((k.decode(), t.value))
            i += 1

    def floats(self, key):
        et = I()
        n = lib().gb_gguf_array_len(self.h, key.encode(), C.byref(et))
        return [lib().gb_gguf_array_float(self.h, key.encode(), j) for j in range(n)]

    def strings(self, key):
        et = I()
        n = lib().gb_gguf_array_len(self.h, key.encode(), C.byref(et))
        buf = C.create_string_buffer(4096)
        out = []
        for j in range(n):
            _check(lib().gb_gguf_array_string(self.h, key.encode(), j, buf, 4096))
            out.append(buf.value.decode())
        return out

    def tensor(self, name):
        t, nd, off, nb, dp = I(), I(), U64(), U64(), P()
        dims = (U64 * 4)()
        rc = lib().gb_gguf_tensor(self.h, name.encode(), C.byref(t), C.byref(nd), dims, C.byref(off),
                                  C.byref(nb), C.byref(dp))
        if rc != OK:
            return None
        data = bytes((C.c_uint8 * nb.value).from_address(dp.value)) if nb.value else b""
        return {"type": t.value, "dims": list(dims[:nd.value]), "offset": off.value, "bytes": nb.value,
                "data": data}

    def close(self):
        if self.h:
            lib().gb_gguf_close(self.h)
            self.h = None
