/*
 * synth.c -- the seeded synthetic inputs of the benchmark, generated on the
 * oracle's side.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). The reference's CPU arm of
 * bench.py and the parity checks need the same synthetic GGUF models the
 * B200 path decodes; this file builds them without loading the product
 * library, so the timed reference arm runs on the oracle alone. It states
 * the generator's rules (not the reference's arithmetic):
 *
 *   every draw comes from a splitmix64 stream keyed by (seed, tensor index,
 *   block index); normals are Box-Muller in float64; per ggml block
 *     Q4_0: d = f16(|N(0,s)|/8), 16 uniform quant bytes
 *     Q8_0: d = f16(|N(0,s)|/128), 32 uniform quant bytes
 *     Q4_K: d, dmin = f16(|N(0,s)|), 140 uniform bytes (scales, quants)
 *     Q5_K: d, dmin = f16(|N(0,s)|), 172 uniform bytes
 *     Q6_K: 192 uniform bytes (ql, qh), 16 int8 scales in [-32, 31],
 *           d = f16(|N(0,s)|)
 *     F16 : one element N(0,s) per block; F32 norms: 1 + N(0, 0.01)
 *   tensors in the order of a llama GGUF (token_embd, per layer attn_norm,
 *   q, k, v, output, ffn_norm, gate, up, down; output_norm, output), written
 *   as a GGUF v3 image (gguf/writer.go:141 layout, alignment 32).
 *
 * tests/test_oracle_synth.py checks that every image and KV fill is byte for
 * byte the one the product library's generator writes.
 */
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "oracle.h"

static uint64_t splitmix64(uint64_t *s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t mix64(uint64_t z) { return splitmix64(&z); }

static uint64_t stream_seed(uint64_t seed, uint64_t tensor, uint64_t block) {
  return mix64(mix64(mix64(seed) ^ tensor) ^ block);
}

static double rng_uniform(uint64_t *s) { return (double)(splitmix64(s) >> 11) * (1.0 / 9007199254740992.0); }

static double rng_normal(uint64_t *s) {
  double u1 = ((double)(splitmix64(s) >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0, 1] */
  double u2 = rng_uniform(s);
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static void rng_bytes(uint64_t *s, uint8_t *p, int n) {
  for (int i = 0; i < n; i += 8) {
    uint64_t v = splitmix64(s);
    for (int j = 0; j < 8 && i + j < n; j++) p[i + j] = (uint8_t)(v >> (8 * j));
  }
}

static void put16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}

static void gen_block(int typ, uint64_t seed, uint32_t tensor, uint64_t block, float sigma, uint8_t *p) {
  uint64_t s = stream_seed(seed, tensor, block);
  switch (typ) {
    case OR_Q4_0:
      put16(p, or_f16_from((float)(fabs(rng_normal(&s) * sigma) / 8.0)));
      rng_bytes(&s, p + 2, 16);
      break;
    case OR_Q8_0:
      put16(p, or_f16_from((float)(fabs(rng_normal(&s) * sigma) / 128.0)));
      rng_bytes(&s, p + 2, 32);
      break;
    case OR_F16:
      put16(p, or_f16_from((float)(rng_normal(&s) * sigma)));
      break;
    case OR_Q4_K:
      put16(p, or_f16_from((float)fabs(rng_normal(&s) * sigma)));
      put16(p + 2, or_f16_from((float)fabs(rng_normal(&s) * sigma)));
      rng_bytes(&s, p + 4, 140);
      break;
    case OR_Q5_K:
      put16(p, or_f16_from((float)fabs(rng_normal(&s) * sigma)));
      put16(p + 2, or_f16_from((float)fabs(rng_normal(&s) * sigma)));
      rng_bytes(&s, p + 4, 172);
      break;
    case OR_Q6_K:
      rng_bytes(&s, p, 192);
      for (int i = 0; i < 16; i++) p[192 + i] = (uint8_t)(int8_t)((int)(splitmix64(&s) % 64) - 32);
      put16(p + 208, or_f16_from((float)fabs(rng_normal(&s) * sigma)));
      break;
    case OR_F32: {
      float v = (float)(1.0 + rng_normal(&s) * sigma);
      memcpy(p, &v, 4);
      break;
    }
  }
}

static int host_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  const char *e = getenv("GB_HOST_THREADS");
  if (e) n = atol(e);
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

typedef struct {
  int typ;
  int64_t b0, b1;
  uint64_t seed;
  uint32_t tensor;
  float sigma;
  uint8_t *dst;
} FillJob;

static void *fill_worker(void *arg) {
  FillJob *j = (FillJob *)arg;
  const int ts = or_type_size(j->typ);
  for (int64_t b = j->b0; b < j->b1; b++) gen_block(j->typ, j->seed, j->tensor, (uint64_t)b, j->sigma, j->dst + b * ts);
  return NULL;
}

static void fill_tensor(int typ, int64_t nblocks, uint64_t seed, uint32_t tensor, float sigma, uint8_t *dst) {
  int nt = host_threads();
  if (nblocks / 64 < nt) nt = (int)(nblocks / 64 > 1 ? nblocks / 64 : 1);
  FillJob jobs[256];
  pthread_t th[256];
  for (int t = 0; t < nt; t++) {
    jobs[t] = (FillJob){typ, nblocks * t / nt, nblocks * (t + 1) / nt, seed, tensor, sigma, dst};
    if (nt == 1) {
      fill_worker(&jobs[t]);
      return;
    }
    pthread_create(&th[t], NULL, fill_worker, &jobs[t]);
  }
  for (int t = 0; t < nt; t++) pthread_join(th[t], NULL);
}

/* ---- the model's tensor list --------------------------------------------- */
typedef struct {
  char name[64];
  int ndims;
  int shape[2]; /* row-major */
  int type;
  float sigma;
} TSpec;

static int quant_type(const or_synth_spec *s, int six) {
  switch (s->mix) {
    case 0: return OR_Q4_0;
    case 2: return OR_Q4_K;
    case 3: return OR_Q6_K;
    case 4: return OR_Q8_0;
    case 5: return OR_F16;
    case 6: return six ? OR_Q6_K : OR_Q5_K;
  }
  return six ? OR_Q6_K : OR_Q4_K;
}

static float model_sigma(int t) {
  if (t == OR_Q4_0 || t == OR_Q8_0 || t == OR_F16) return 0.02f;
  if (t == OR_Q4_K) return 0.01f / 128.f;
  if (t == OR_Q5_K) return 0.01f / 256.f;
  return 0.002f / 32.f;
}

static void add_mat(TSpec *v, int *n, const char *name, int rows, int cols, int type) {
  TSpec *t = &v[(*n)++];
  snprintf(t->name, sizeof t->name, "%s", name);
  t->ndims = 2;
  t->shape[0] = rows;
  t->shape[1] = cols;
  t->type = type;
  t->sigma = model_sigma(type);
}

static void add_vec(TSpec *v, int *n, const char *name, int len) {
  TSpec *t = &v[(*n)++];
  snprintf(t->name, sizeof t->name, "%s", name);
  t->ndims = 1;
  t->shape[0] = len;
  t->shape[1] = 1;
  t->type = OR_F32;
  t->sigma = 0.01f;
}

static int model_tensors(const or_synth_spec *s, TSpec *v) {
  int n = 0;
  const int kv_dim = s->kv_heads * s->head_dim, q_dim = s->heads * s->head_dim;
  char nm[64];
  add_mat(v, &n, "token_embd.weight", s->vocab, s->dim, quant_type(s, 0));
  for (int i = 0; i < s->layers; i++) {
#define NAME(suffix) (snprintf(nm, sizeof nm, "blk.%d.%s", i, suffix), nm)
    add_vec(v, &n, NAME("attn_norm.weight"), s->dim);
    add_mat(v, &n, NAME("attn_q.weight"), q_dim, s->dim, quant_type(s, 0));
    add_mat(v, &n, NAME("attn_k.weight"), kv_dim, s->dim, quant_type(s, 0));
    add_mat(v, &n, NAME("attn_v.weight"), kv_dim, s->dim, quant_type(s, 1));
    add_mat(v, &n, NAME("attn_output.weight"), s->dim, q_dim, quant_type(s, 0));
    add_vec(v, &n, NAME("ffn_norm.weight"), s->dim);
    add_mat(v, &n, NAME("ffn_gate.weight"), s->ffn, s->dim, quant_type(s, 0));
    add_mat(v, &n, NAME("ffn_up.weight"), s->ffn, s->dim, quant_type(s, 0));
    add_mat(v, &n, NAME("ffn_down.weight"), s->dim, s->ffn, quant_type(s, i % 2 == 0));
#undef NAME
  }
  add_vec(v, &n, "output_norm.weight", s->dim);
  if (s->mix != 0) add_mat(v, &n, "output.weight", s->vocab, s->dim, quant_type(s, 1));
  return n;
}

/* ---- GGUF v3 bytes (gguf/writer.go:141 layout) ---------------------------- */
typedef struct {
  uint8_t *b;
  size_t n, cap;
} Buf;

static void put(Buf *o, const void *p, size_t n) {
  if (o->n + n > o->cap) {
    o->cap = (o->n + n) * 2 + 256;
    o->b = (uint8_t *)realloc(o->b, o->cap);
  }
  memcpy(o->b + o->n, p, n);
  o->n += n;
}
static void le(Buf *o, uint64_t v, int n) {
  uint8_t t[8];
  for (int i = 0; i < n; i++) t[i] = (uint8_t)(v >> (8 * i));
  put(o, t, (size_t)n);
}
static void str(Buf *o, const char *s) {
  le(o, strlen(s), 8);
  put(o, s, strlen(s));
}
static void kv_u32(Buf *o, const char *k, uint32_t v) {
  str(o, k);
  le(o, 4, 4);
  le(o, v, 4);
}
static void kv_f32(Buf *o, const char *k, float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  str(o, k);
  le(o, 6, 4);
  le(o, u, 4);
}
static void kv_str(Buf *o, const char *k, const char *v) {
  str(o, k);
  le(o, 8, 4);
  str(o, v);
}

int or_synth_preset(int preset, or_synth_spec *s) {
  if (!s) return -1;
  memset(s, 0, sizeof *s);
  s->vocab = 128256;
  s->rope_base = 500000.f;
  s->eps = 1e-5f;
  switch (preset) {
    case 1:
      s->layers = 16; s->dim = 2048; s->heads = 32; s->kv_heads = 8; s->head_dim = 64;
      s->ffn = 8192; s->ctx_len = 2048; s->mix = 0;
      break;
    case 3:
      s->layers = 28; s->dim = 3072; s->heads = 24; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 8192; s->ctx_len = 4096; s->mix = 1;
      break;
    case 8:
      s->layers = 32; s->dim = 4096; s->heads = 32; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 14336; s->ctx_len = 8320; s->mix = 1;
      break;
    case 70:
      s->layers = 80; s->dim = 8192; s->heads = 64; s->kv_heads = 8; s->head_dim = 128;
      s->ffn = 28672; s->ctx_len = 8192; s->mix = 1;
      break;
    default:
      return -1;
  }
  return 0;
}

int or_synth_model(const or_synth_spec *s, uint8_t **out, size_t *out_len) {
  if (!s || !out || !out_len || s->layers <= 0 || s->dim <= 0 || s->ffn <= 0 || s->heads <= 0 ||
      s->kv_heads <= 0 || s->head_dim <= 0 || s->vocab <= 0 || s->heads % s->kv_heads != 0)
    return -1;
  const int max_t = 9 * s->layers + 3;
  TSpec *ts = (TSpec *)calloc((size_t)max_t, sizeof(TSpec));
  if (!ts) return -2;
  const int nt = model_tensors(s, ts);
  Buf o = {0};
  int nkv = 10 + (s->head_dim != s->dim / s->heads ? 1 : 0);
  le(&o, 0x46554747u, 4);
  le(&o, 3, 4);
  le(&o, (uint64_t)nt, 8);
  le(&o, (uint64_t)nkv, 8);
  kv_str(&o, "general.architecture", "llama");
  kv_str(&o, "general.name", "gollama-b200 synthetic");
  kv_u32(&o, "llama.block_count", (uint32_t)s->layers);
  kv_u32(&o, "llama.embedding_length", (uint32_t)s->dim);
  kv_u32(&o, "llama.feed_forward_length", (uint32_t)s->ffn);
  kv_u32(&o, "llama.attention.head_count", (uint32_t)s->heads);
  kv_u32(&o, "llama.attention.head_count_kv", (uint32_t)s->kv_heads);
  kv_u32(&o, "llama.context_length", (uint32_t)s->ctx_len);
  kv_f32(&o, "llama.rope.freq_base", s->rope_base);
  kv_f32(&o, "llama.attention.layer_norm_rms_epsilon", s->eps);
  if (s->head_dim != s->dim / s->heads) kv_u32(&o, "llama.attention.key_length", (uint32_t)s->head_dim);
  uint64_t *offs = (uint64_t *)calloc((size_t)nt, sizeof(uint64_t));
  uint64_t *bytes = (uint64_t *)calloc((size_t)nt, sizeof(uint64_t));
  uint64_t off = 0;
  const uint64_t align = 32;
  for (int i = 0; i < nt; i++) {
    const TSpec *t = &ts[i];
    str(&o, t->name);
    le(&o, (uint64_t)t->ndims, 4);
    for (int d = t->ndims - 1; d >= 0; d--) le(&o, (uint64_t)t->shape[d], 8); /* innermost first */
    le(&o, (uint64_t)t->type, 4);
    le(&o, off, 8);
    offs[i] = off;
    const int inner = t->shape[t->ndims - 1];
    const uint64_t rows = t->ndims == 2 ? (uint64_t)t->shape[0] : 1;
    bytes[i] = (uint64_t)or_row_bytes(t->type, inner) * rows;
    off = (off + bytes[i] + align - 1) / align * align;
  }
  while (o.n % align) le(&o, 0, 1);
  const size_t hdr = o.n, total = hdr + (size_t)off;
  uint8_t *img = (uint8_t *)malloc(total);
  if (!img) {
    free(o.b);
    free(offs);
    free(bytes);
    free(ts);
    return -2;
  }
  memcpy(img, o.b, hdr);
  free(o.b);
  for (int i = 0; i < nt; i++) {
    const TSpec *t = &ts[i];
    uint8_t *dst = img + hdr + offs[i];
    const uint64_t n = (uint64_t)t->shape[0] * (t->ndims == 2 ? (uint64_t)t->shape[1] : 1);
    fill_tensor(t->type, (int64_t)(n / (uint64_t)or_block_size(t->type)), s->seed, (uint32_t)i, t->sigma, dst);
    const uint64_t end = offs[i] + bytes[i];
    const uint64_t next = i + 1 < nt ? offs[i + 1] : (uint64_t)off;
    memset(img + hdr + end, 0, (size_t)(next - end));
  }
  free(offs);
  free(bytes);
  free(ts);
  *out = img;
  *out_len = total;
  return 0;
}

void or_synth_free(uint8_t *img) { free(img); }

typedef struct {
  uint64_t seed;
  int layer, pos0, kv_dim, f16;
  int64_t i0, i1;
  float *k, *v;
} KvJob;

static void *kv_worker(void *arg) {
  KvJob *j = (KvJob *)arg;
  for (int64_t i = j->i0; i < j->i1; i++) {
    for (int which = 0; which < 2; which++) {
      uint64_t s = stream_seed(j->seed, 0x40000000u + 2u * (uint32_t)j->layer + (uint32_t)which, (uint64_t)(j->pos0 + i));
      float *dst = (which ? j->v : j->k) + i * j->kv_dim;
      for (int d = 0; d < j->kv_dim; d++) {
        float x = (float)rng_normal(&s);
        dst[d] = j->f16 ? or_f16_to_f32(or_f16_from(x)) : x;
      }
    }
  }
  return NULL;
}

int or_synth_kv_normal(uint64_t seed, int layer, int pos0, int n, int kv_dim, int f16, float *k, float *v) {
  if (layer < 0 || pos0 < 0 || n < 0 || kv_dim <= 0 || !k || !v) return -1;
  int nt = host_threads();
  if (n / 64 < nt) nt = n / 64 > 1 ? n / 64 : 1;
  KvJob jobs[256];
  pthread_t th[256];
  for (int t = 0; t < nt; t++) {
    jobs[t] = (KvJob){seed, layer, pos0, kv_dim, f16, (int64_t)n * t / nt, (int64_t)n * (t + 1) / nt, k, v};
    if (nt == 1) {
      kv_worker(&jobs[t]);
      return 0;
    }
    pthread_create(&th[t], NULL, kv_worker, &jobs[t]);
  }
  for (int t = 0; t < nt; t++) pthread_join(th[t], NULL);
  return 0;
}
