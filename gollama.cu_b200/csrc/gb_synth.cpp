// gb_synth.cpp -- seeded synthetic llama GGUF models, matrices and KV fills.
//
// Every random draw comes from a splitmix64 stream keyed by
// (seed, tensor id, block index), so any block can be regenerated on its own
// and the image is identical however many threads build it. Normals are
// Box-Muller in float64. Block recipes (per ggml block):
//   Q4_0: d = f16(|N(0,sigma)|/8), 16 uniform quant bytes            (sigma 0.02)
//   Q4_K: d, dmin = f16(|N(0,sigma)|), 12 uniform scale bytes,
//         128 uniform quant bytes                                      (sigma 0.01)
//   Q5_K: d, dmin = f16(|N(0,sigma)|), 12 scale + 32 qh + 128 qs uniform
//         bytes                                                        (sigma 0.005)
//   Q6_K: 128 ql + 64 qh uniform bytes, 16 int8 scales uniform in
//         [-32,31], d = f16(|N(0,sigma)|)                              (sigma 0.002)
//   norms: float32 1 + N(0, 0.01)
// The sigma values above are the standalone-matrix (GEMV sweep) recipe. The
// Q4_K / Q6_K model presets divide sigma by 128 and 32 so that weights have
// an rms near 0.02, like a trained llama, and activations stay O(1) through
// every layer.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>

#include "gb_internal.h"

uint64_t gb_splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t mix64(uint64_t z) {
  uint64_t s = z;
  return gb_splitmix64(&s);
}

uint64_t gb_stream_seed(uint64_t seed, uint64_t tensor, uint64_t block) {
  return mix64(mix64(mix64(seed) ^ tensor) ^ block);
}

int gb_host_threads() {
  unsigned n = std::thread::hardware_concurrency();
  if (const char *e = getenv("GB_HOST_THREADS")) n = (unsigned)atoi(e);
  return n < 1 ? 1 : (int)std::min(n, 256u);
}

namespace {

struct Rng {
  uint64_t s;
  uint64_t next() { return gb_splitmix64(&s); }
  double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
  double normal() {
    double u1 = ((double)(next() >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0,1]
    double u2 = uniform();
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
  }
  void bytes(uint8_t *p, int n) {
    for (int i = 0; i < n; i += 8) {
      uint64_t v = next();
      for (int j = 0; j < 8 && i + j < n; j++) p[i + j] = (uint8_t)(v >> (8 * j));
    }
  }
};

// binary16 round-to-nearest-even of a float (f16.From, f16/f16.go:11).
uint16_t f16_from(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  uint16_t sign = (uint16_t)(b >> 16) & 0x8000;
  int32_t exp = (int32_t)((b >> 23) & 0xff) - 127;
  uint32_t mant = b & 0x7fffff;
  if (exp == 128) return mant ? (uint16_t)(sign | 0x7e00) : (uint16_t)(sign | 0x7c00);
  if (exp > 15) return (uint16_t)(sign | 0x7c00);
  if (exp >= -14) {
    uint32_t m = mant >> 13, rem = mant & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (m & 1))) m++;
    return (uint16_t)((uint16_t)(sign | (uint16_t)((uint32_t)(exp + 15) << 10)) + (uint16_t)m);
  }
  if (exp >= -25) {
    uint32_t full = mant | 0x800000, shift = (uint32_t)(-exp - 1);
    uint32_t m = full >> shift, rem = full & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1))) m++;
    return (uint16_t)(sign | (uint16_t)m);
  }
  return sign;
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1f, mant = h & 0x3ff, b;
  if (exp == 0) {
    if (mant == 0) {
      b = sign;
    } else {
      uint32_t e = 127 - 15 + 1;
      while (!(mant & 0x400)) { mant <<= 1; e--; }
      b = sign | e << 23 | (mant & 0x3ff) << 13;
    }
  } else if (exp == 0x1f) {
    b = sign | 0x7f800000 | mant << 13;
  } else {
    b = sign | (exp + 127 - 15) << 23 | mant << 13;
  }
  float f;
  memcpy(&f, &b, 4);
  return f;
}

void put16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}

// One ggml block of typ, drawn from its own stream.
void gen_block(int typ, uint64_t seed, uint32_t tensor, uint64_t block, float sigma, uint8_t *p) {
  Rng r{gb_stream_seed(seed, tensor, block)};
  switch (typ) {
    case GB_T_Q4_0:
      put16(p, f16_from((float)(fabs(r.normal() * sigma) / 8.0)));
      r.bytes(p + 2, 16);
      break;
    case GB_T_Q8_0:
      put16(p, f16_from((float)(fabs(r.normal() * sigma) / 128.0)));
      r.bytes(p + 2, 32);
      break;
    case GB_T_F16:  // one element per "block": N(0, sigma)
      put16(p, f16_from((float)(r.normal() * sigma)));
      break;
    case GB_T_Q4_K:
      put16(p, f16_from((float)fabs(r.normal() * sigma)));
      put16(p + 2, f16_from((float)fabs(r.normal() * sigma)));
      r.bytes(p + 4, 140);
      break;
    case GB_T_Q5_K:
      put16(p, f16_from((float)fabs(r.normal() * sigma)));
      put16(p + 2, f16_from((float)fabs(r.normal() * sigma)));
      r.bytes(p + 4, 172);
      break;
    case GB_T_Q6_K:
      r.bytes(p, 192);
      for (int i = 0; i < 16; i++) p[192 + i] = (uint8_t)(int8_t)((int)(r.next() % 64) - 32);
      put16(p + 208, f16_from((float)fabs(r.normal() * sigma)));
      break;
    case GB_T_F32:  // one element per "block": 1 + N(0, sigma)
    {
      float v = (float)(1.0 + r.normal() * sigma);
      memcpy(p, &v, 4);
      break;
    }
  }
}

template <class F>
void parallel_for(int64_t n, F f) {
  int nt = (int)std::min<int64_t>(gb_host_threads(), std::max<int64_t>(1, n / 64));
  if (nt <= 1) {
    for (int64_t i = 0; i < n; i++) f(i);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < nt; t++)
    th.emplace_back([=] {
      for (int64_t i = n * t / nt; i < n * (t + 1) / nt; i++) f(i);
    });
  for (auto &x : th) x.join();
}

void fill_tensor(int typ, int64_t nblocks, uint64_t seed, uint32_t tensor, float sigma,
                 uint8_t *dst) {
  int ts = gb_type_size(typ);
  parallel_for(nblocks, [&](int64_t b) { gen_block(typ, seed, tensor, (uint64_t)b, sigma, dst + b * ts); });
}

float default_sigma(int typ) {
  switch (typ) {
    case GB_T_Q4_0: return 0.02f;
    case GB_T_Q8_0: return 0.02f;
    case GB_T_F16: return 0.02f;
    case GB_T_Q4_K: return 0.01f;
    case GB_T_Q5_K: return 0.005f;
    case GB_T_Q6_K: return 0.002f;
  }
  return 0.01f;
}

struct TensorSpec {
  std::string name;
  std::vector<int> shape;
  int type;
  float sigma;
};

std::vector<TensorSpec> model_tensors(const gb_synth_spec &s) {
  std::vector<TensorSpec> v;
  int kv_dim = s.kv_heads * s.head_dim, q_dim = s.heads * s.head_dim;
  auto qt = [&](bool six) {
    if (s.mix == 0) return (int)GB_T_Q4_0;
    if (s.mix == 2) return (int)GB_T_Q4_K;
    if (s.mix == 3) return (int)GB_T_Q6_K;
    if (s.mix == 4) return (int)GB_T_Q8_0;
    if (s.mix == 5) return (int)GB_T_F16;
    if (s.mix == 6) return six ? (int)GB_T_Q6_K : (int)GB_T_Q5_K;  // Q5_K_M
    return six ? (int)GB_T_Q6_K : (int)GB_T_Q4_K;
  };
  auto sig = [&](int t) {
    if (t == GB_T_Q4_0 || t == GB_T_Q8_0) return 0.02f;
    if (t == GB_T_F16) return 0.02f;
    if (t == GB_T_Q4_K) return 0.01f / 128.f;
    if (t == GB_T_Q5_K) return 0.01f / 256.f;  // 5-bit quants: twice the range of Q4_K's
    return 0.002f / 32.f;
  };
  auto mat = [&](const std::string &n, int rows, int cols, bool six) {
    int t = qt(six);
    v.push_back({n, {rows, cols}, t, sig(t)});
  };
  mat("token_embd.weight", s.vocab, s.dim, false);
  for (int i = 0; i < s.layers; i++) {
    std::string p = "blk." + std::to_string(i) + ".";
    v.push_back({p + "attn_norm.weight", {s.dim}, GB_T_F32, 0.01f});
    mat(p + "attn_q.weight", q_dim, s.dim, false);
    mat(p + "attn_k.weight", kv_dim, s.dim, false);
    mat(p + "attn_v.weight", kv_dim, s.dim, true);
    mat(p + "attn_output.weight", s.dim, q_dim, false);
    v.push_back({p + "ffn_norm.weight", {s.dim}, GB_T_F32, 0.01f});
    mat(p + "ffn_gate.weight", s.ffn, s.dim, false);
    mat(p + "ffn_up.weight", s.ffn, s.dim, false);
    mat(p + "ffn_down.weight", s.dim, s.ffn, i % 2 == 0);  // Q4_K_M: even layers Q6_K
  }
  v.push_back({"output_norm.weight", {s.dim}, GB_T_F32, 0.01f});
  if (s.mix != 0) mat("output.weight", s.vocab, s.dim, true);  // mix 0: tied to token_embd
  return v;
}

int build_image(const gb_synth_spec &s, uint8_t **out, size_t *out_len) {
  if (s.layers <= 0 || s.dim <= 0 || s.ffn <= 0 || s.heads <= 0 || s.kv_heads <= 0 ||
      s.head_dim <= 0 || s.vocab <= 0 || s.heads % s.kv_heads != 0)
    return gb_fail(GB_ERR_INVALID, "synth: invalid model shape");
  GbGgufWriter w;
  w.set_str("general.architecture", "llama");
  w.set_str("general.name", "gollama-b200 synthetic");
  w.set_u32("llama.block_count", (uint32_t)s.layers);
  w.set_u32("llama.embedding_length", (uint32_t)s.dim);
  w.set_u32("llama.feed_forward_length", (uint32_t)s.ffn);
  w.set_u32("llama.attention.head_count", (uint32_t)s.heads);
  w.set_u32("llama.attention.head_count_kv", (uint32_t)s.kv_heads);
  w.set_u32("llama.context_length", (uint32_t)s.ctx_len);
  w.set_f32("llama.rope.freq_base", s.rope_base);
  w.set_f32("llama.attention.layer_norm_rms_epsilon", s.eps);
  if (s.head_dim != s.dim / s.heads) w.set_u32("llama.attention.key_length", (uint32_t)s.head_dim);
  auto specs = model_tensors(s);
  for (auto &t : specs) {
    int rc = w.add_tensor(t.name, t.shape, t.type, std::vector<uint8_t>());
    if (rc) return rc;
  }
  std::vector<uint64_t> offs;
  uint64_t total = 0;
  std::vector<uint8_t> hdr = w.layout(&offs, &total);
  uint8_t *img = (uint8_t *)malloc((size_t)total);
  if (!img) return gb_fail(GB_ERR_INVALID, "synth: cannot allocate %llu bytes", (unsigned long long)total);
  memcpy(img, hdr.data(), hdr.size());
  for (size_t i = 0; i < specs.size(); i++) {
    const auto &t = specs[i];
    uint8_t *dst = img + hdr.size() + offs[i];
    uint64_t n = 1;
    for (int d : t.shape) n *= (uint64_t)d;
    int64_t nblocks = (int64_t)(n / (uint64_t)gb_block_size(t.type));
    fill_tensor(t.type, nblocks, s.seed, (uint32_t)i, t.sigma, dst);
    uint64_t end = offs[i] + w.tensors[i].bytes;
    uint64_t next = i + 1 < specs.size() ? offs[i + 1] : total - hdr.size();
    memset(img + hdr.size() + end, 0, (size_t)(next - end));
  }
  *out = img;
  *out_len = (size_t)total;
  return GB_OK;
}

}  // namespace

extern "C" {

int gb_synth_preset(int preset, gb_synth_spec *s) {
  gb_clear_error();
  if (!s) return gb_fail(GB_ERR_INVALID, "synth: null spec");
  memset(s, 0, sizeof *s);
  s->vocab = 128256;
  s->rope_base = 500000.f;
  s->eps = 1e-5f;
  s->seed = 0;
  switch (preset) {
    case 1:  // Llama-3.2-1B shape, Q4_0, tied head
      s->layers = 16; s->dim = 2048; s->heads = 32; s->kv_heads = 8; s->head_dim = 64;
      s->ffn = 8192; s->ctx_len = 2048; s->mix = 0;
      break;
    case 3:  // Llama-3.2-3B shape, Q4_K_M
      s->layers = 28; s->dim = 3072; s->heads = 24; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 8192; s->ctx_len = 4096; s->mix = 1;
      break;
    case 8:  // Llama-3.1-8B shape, Q4_K_M; context covers 8192 prefilled + 128 decode
      s->layers = 32; s->dim = 4096; s->heads = 32; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 14336; s->ctx_len = 8320; s->mix = 1;
      break;
    case 70:  // Llama-3.1-70B shape, Q4_K_M
      s->layers = 80; s->dim = 8192; s->heads = 64; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 28672; s->ctx_len = 8192; s->mix = 1;
      break;
    default:
      return gb_fail(GB_ERR_INVALID, "synth: unknown preset %d", preset);
  }
  return GB_OK;
}

int gb_synth_model(const gb_synth_spec *spec, void **gguf, size_t *len) {
  gb_clear_error();
  if (!spec || !gguf || !len) return gb_fail(GB_ERR_INVALID, "synth: null argument");
  uint8_t *img = nullptr;
  int rc = build_image(*spec, &img, len);
  if (rc) return rc;
  *gguf = img;
  return GB_OK;
}

int gb_synth_model_file(const gb_synth_spec *spec, const char *path) {
  gb_clear_error();
  uint8_t *img = nullptr;
  size_t len = 0;
  int rc = build_image(*spec, &img, &len);
  if (rc) return rc;
  FILE *f = fopen(path, "wb");
  if (!f) {
    free(img);
    return gb_fail(GB_ERR_IO, "synth: cannot create %s", path);
  }
  size_t wr = fwrite(img, 1, len, f);
  int cl = fclose(f);
  free(img);
  if (wr != len || cl != 0) return gb_fail(GB_ERR_IO, "synth: short write to %s", path);
  return GB_OK;
}

void gb_synth_free(void *gguf) { free(gguf); }

int gb_synth_matrix(int typ, int rows, int cols, uint64_t seed, uint32_t tensor_id,
                    float scale_sigma, void *buf) {
  gb_clear_error();
  if (!gb_tiled_type(typ) || rows <= 0 || cols <= 0 || cols % gb_block_size(typ) || !buf)
    return gb_fail(GB_ERR_INVALID, "synth: bad matrix request");
  int64_t nblocks = (int64_t)rows * (cols / gb_block_size(typ));
  fill_tensor(typ, nblocks, seed, tensor_id, scale_sigma > 0 ? scale_sigma : default_sigma(typ),
              (uint8_t *)buf);
  return GB_OK;
}

int gb_synth_normal(uint64_t seed, uint32_t stream_id, int64_t n, float *out) {
  gb_clear_error();
  if (n < 0 || (n > 0 && !out)) return gb_fail(GB_ERR_INVALID, "synth: bad normal request");
  const int64_t chunk = 1024;
  parallel_for((n + chunk - 1) / chunk, [&](int64_t c) {
    Rng r{gb_stream_seed(seed, 0x80000000u | stream_id, (uint64_t)c)};
    for (int64_t i = c * chunk; i < std::min(n, (c + 1) * chunk); i++) out[i] = (float)r.normal();
  });
  return GB_OK;
}

int gb_synth_kv_normal(uint64_t seed, int layer, int pos0, int n, int kv_dim, int f16, float *k,
                       float *v) {
  gb_clear_error();
  if (layer < 0 || pos0 < 0 || n < 0 || kv_dim <= 0 || !k || !v)
    return gb_fail(GB_ERR_INVALID, "synth: bad KV request");
  parallel_for(n, [&](int64_t i) {
    for (int which = 0; which < 2; which++) {
      Rng r{gb_stream_seed(seed, 0x40000000u + 2u * (uint32_t)layer + (uint32_t)which,
                           (uint64_t)(pos0 + i))};
      float *dst = (which ? v : k) + i * kv_dim;
      for (int j = 0; j < kv_dim; j++) {
        float x = (float)r.normal();
        dst[j] = f16 ? f16_to_f32(f16_from(x)) : x;
      }
    }
  });
  return GB_OK;
}

}  // extern "C"
