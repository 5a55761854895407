/*
 * oracle.c -- CPU restatement of gollama.cu's pure-Go reference path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Each function cites the Go
 * function it restates, by file:line in the reference project. Built with
 * -ffp-contract=off so that float32 expressions round after every
 * operation, as Go does on amd64.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- types (gguf/types.go:47-81) ---------------------------------------- */

int or_block_size(int typ) {
  switch (typ) {
    case OR_F32: case OR_F16: case OR_BF16: return 1;
    case 24: case 25: case 26: case 27: case 28: return 1; /* I8..F64 */
    case OR_Q4_0: case 3: case 6: case 7: case OR_Q8_0: case 9: case 20: return 32;
    case 10: case 11: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: case 15:
    case 16: case 17: case 18: case 19: case 21: case 22: case 23: case 29: return 256;
  }
  return 0;
}

int or_type_size(int typ) {
  switch (typ) {
    case OR_F32: return 4;  case OR_F16: return 2;  case OR_BF16: return 2; case 28: return 8;
    case 24: return 1;      case 25: return 2;      case 26: return 4;      case 27: return 8;
    case OR_Q4_0: return 18; case 3: return 20;     case 6: return 22;      case 7: return 24;
    case OR_Q8_0: return 34; case 9: return 36;
    case 10: return 84;     case 11: return 110;    case OR_Q4_K: return 144;
    case OR_Q5_K: return 176; case OR_Q6_K: return 210; case 15: return 292;
    case 16: return 66;     case 17: return 74;     case 18: return 98;     case 19: return 50;
    case 20: return 18;     case 21: return 110;    case 22: return 82;     case 23: return 136;
    case 29: return 56;
  }
  return 0;
}

int64_t or_row_bytes(int typ, int64_t n) {
  int bs = or_block_size(typ);
  return bs ? n / bs * or_type_size(typ) : 0;
}

/* ---- binary16 (f16/f16.go:11-69) ---------------------------------------- */

static uint32_t f32_bits(float x) { uint32_t b; memcpy(&b, &x, 4); return b; }
static float f32_from_bits(uint32_t b) { float x; memcpy(&x, &b, 4); return x; }

/* f16/f16.go:11 From. */
uint16_t or_f16_from(float x) {
  uint32_t b = f32_bits(x);
  uint16_t sign = (uint16_t)(b >> 16) & 0x8000;
  int32_t exp = (int32_t)((b >> 23) & 0xff) - 127;
  uint32_t mant = b & 0x7fffff;
  if (exp == 128) return mant != 0 ? (uint16_t)(sign | 0x7e00) : (uint16_t)(sign | 0x7c00);
  if (exp > 15) return (uint16_t)(sign | 0x7c00);
  if (exp >= -14) {
    uint32_t m = mant >> 13, rem = mant & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (m & 1) == 1)) m++;
    return (uint16_t)((uint16_t)(sign | (uint16_t)((uint32_t)(exp + 15) << 10)) + (uint16_t)m);
  }
  if (exp >= -25) {
    uint32_t full = mant | 0x800000;
    uint32_t shift = (uint32_t)(-exp - 1);
    uint32_t m = full >> shift, rem = full & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (m & 1) == 1)) m++;
    return (uint16_t)(sign | (uint16_t)m);
  }
  return sign;
}

/* f16/f16.go:47 Float32. */
float or_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
  if (exp == 0) {
    if (mant == 0) return f32_from_bits(sign);
    uint32_t e = 127 - 15 + 1;
    while ((mant & 0x400) == 0) { mant <<= 1; e--; }
    mant &= 0x3ff;
    return f32_from_bits(sign | e << 23 | mant << 13);
  }
  if (exp == 0x1f) return f32_from_bits(sign | 0x7f800000 | mant << 13);
  return f32_from_bits(sign | (exp + 127 - 15) << 23 | mant << 13);
}

/* ---- dequantization (quant/quant.go:27-138) ----------------------------- */

static float half_at(const uint8_t *b) { return or_f16_to_f32((uint16_t)(b[0] | b[1] << 8)); }

/* quant/quant.go:90 ScaleMinQ4K (ggml get_scale_min_k4). */
void or_scale_min_q4k(const uint8_t *s, int j, uint8_t *sc, uint8_t *m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* quant/quant.go:97 dequantQ4K. */
static void dequant_q4k(const uint8_t *blk, float *out) {
  float d = half_at(blk), dmin = half_at(blk + 2);
  const uint8_t *scales = blk + 4, *q = blk + 16;
  for (int chunk = 0; chunk < 4; chunk++) {
    uint8_t sc1, m1, sc2, m2;
    or_scale_min_q4k(scales, 2 * chunk, &sc1, &m1);
    or_scale_min_q4k(scales, 2 * chunk + 1, &sc2, &m2);
    float d1 = d * (float)sc1, min1 = dmin * (float)m1;
    float d2 = d * (float)sc2, min2 = dmin * (float)m2;
    const uint8_t *qs = q + chunk * 32;
    float *y = out + chunk * 64;
    for (int l = 0; l < 32; l++) {
      y[l] = d1 * (float)(qs[l] & 0xF) - min1;
      y[l + 32] = d2 * (float)(qs[l] >> 4) - min2;
    }
  }
}

/* Q5_K. The reference lists the type (gguf/types.go:53: 256 elements in 176
 * bytes) but quant.Dequantize has no case for it; this restates the published
 * ggml block_q5_K layout: d and dmin (binary16), 12 scale bytes packed as for
 * Q4_K, qh[32] holding the fifth bits, qs[128] the low four. Element 64j + l
 * of the block is (d*sc)*q - dmin*m of sub-block 2j with
 * q = (qs[32j+l] & 15) | bit 2j of qh[l] << 4, element 64j + 32 + l the same
 * with the high nibble, bit 2j+1 and sub-block 2j+1 (float32 as dequantQ4K). */
static void dequant_q5k(const uint8_t *blk, float *out) {
  float d = half_at(blk), dmin = half_at(blk + 2);
  const uint8_t *scales = blk + 4, *qh = blk + 16, *q = blk + 48;
  for (int chunk = 0; chunk < 4; chunk++) {
    uint8_t sc1, m1, sc2, m2;
    or_scale_min_q4k(scales, 2 * chunk, &sc1, &m1);
    or_scale_min_q4k(scales, 2 * chunk + 1, &sc2, &m2);
    float d1 = d * (float)sc1, min1 = dmin * (float)m1;
    float d2 = d * (float)sc2, min2 = dmin * (float)m2;
    const uint8_t *qs = q + chunk * 32;
    float *y = out + chunk * 64;
    for (int l = 0; l < 32; l++) {
      int lo = (qs[l] & 0xF) | (((qh[l] >> (2 * chunk)) & 1) << 4);
      int hi = (qs[l] >> 4) | (((qh[l] >> (2 * chunk + 1)) & 1) << 4);
      y[l] = d1 * (float)lo - min1;
      y[l + 32] = d2 * (float)hi - min2;
    }
  }
}

/* quant/quant.go:114 dequantQ6K. */
static void dequant_q6k(const uint8_t *blk, float *out) {
  const uint8_t *ql = blk, *qh = blk + 128;
  const int8_t *sc = (const int8_t *)(blk + 192);
  float d = half_at(blk + 208);
  for (int chunk = 0; chunk < 2; chunk++) {
    const uint8_t *l0 = ql + chunk * 64, *h0 = qh + chunk * 32;
    const int8_t *s0 = sc + chunk * 8;
    float *y = out + chunk * 128;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      int8_t q1 = (int8_t)((l0[l] & 0xF) | (((h0[l] >> 0) & 3) << 4)) - 32;
      int8_t q2 = (int8_t)((l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4)) - 32;
      int8_t q3 = (int8_t)((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32;
      int8_t q4 = (int8_t)((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * (float)s0[is] * (float)q1;
      y[l + 32] = d * (float)s0[is + 2] * (float)q2;
      y[l + 64] = d * (float)s0[is + 4] * (float)q3;
      y[l + 96] = d * (float)s0[is + 6] * (float)q4;
    }
  }
}

/* quant/quant.go:27 Dequantize. */
int or_dequantize(int typ, const uint8_t *data, int64_t len, float *out, int64_t n) {
  int bs = or_block_size(typ);
  if (bs == 0) return -3;
  if (n % bs != 0) return -1;
  if (len < or_row_bytes(typ, n)) return -2;
  switch (typ) {
    case OR_F32:
      for (int64_t i = 0; i < n; i++) out[i] = f32_from_bits((uint32_t)data[4 * i] |
          (uint32_t)data[4 * i + 1] << 8 | (uint32_t)data[4 * i + 2] << 16 | (uint32_t)data[4 * i + 3] << 24);
      return 0;
    case OR_F16:
      for (int64_t i = 0; i < n; i++) out[i] = half_at(data + 2 * i);
      return 0;
    case OR_BF16:
      for (int64_t i = 0; i < n; i++)
        out[i] = f32_from_bits((uint32_t)(data[2 * i] | data[2 * i + 1] << 8) << 16);
      return 0;
    case OR_Q8_0:
      for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 34;
        float d = half_at(blk);
        for (int j = 0; j < 32; j++) out[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
      }
      return 0;
    case OR_Q4_0:
      for (int64_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 18;
        float d = half_at(blk);
        for (int j = 0; j < 16; j++) {
          uint8_t q = blk[2 + j];
          out[b * 32 + j] = d * ((float)(q & 0xF) - 8);
          out[b * 32 + j + 16] = d * ((float)(q >> 4) - 8);
        }
      }
      return 0;
    case OR_Q4_K:
      for (int64_t b = 0; b < n / 256; b++) dequant_q4k(data + b * 144, out + b * 256);
      return 0;
    case OR_Q5_K:
      for (int64_t b = 0; b < n / 256; b++) dequant_q5k(data + b * 176, out + b * 256);
      return 0;
    case OR_Q6_K:
      for (int64_t b = 0; b < n / 256; b++) dequant_q6k(data + b * 210, out + b * 256);
      return 0;
  }
  return -3;
}

/* quant/quant.go:135 Row. */
int or_row(int typ, const uint8_t *data, int64_t len, int cols, int64_t r, float *out) {
  int64_t rb = or_row_bytes(typ, cols);
  if (rb <= 0 || (r + 1) * rb > len) return -2;
  return or_dequantize(typ, data + r * rb, rb, out, cols);
}

/* ---- backend/cpu/cpu.go ------------------------------------------------- */

/* backend/cpu/cpu.go:17 RMSNorm. */
void or_rmsnorm(const float *x, const float *w, float *out, int rows, int n, float eps) {
  for (int r = 0; r < rows; r++) {
    const float *xr = x + (int64_t)r * n;
    float *o = out + (int64_t)r * n;
    double ss = 0;
    for (int i = 0; i < n; i++) ss += (double)xr[i] * (double)xr[i];
    float inv = (float)(1 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; i++) o[i] = xr[i] * inv * w[i];
  }
}

/* Go's builtin max for floats: NaN if either is NaN, +0 over -0. */
static float go_max(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == 0 && b == 0) return signbit(a) ? b : a;
  return a > b ? a : b;
}

/* backend/cpu/cpu.go:32 Softmax. */
void or_softmax(const float *x, float *out, int rows, int n) {
  for (int r = 0; r < rows; r++) {
    const float *xr = x + (int64_t)r * n;
    float *o = out + (int64_t)r * n;
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = go_max(m, xr[i]);
    double sum = 0;
    for (int i = 0; i < n; i++) {
      float e = (float)exp((double)(xr[i] - m));
      o[i] = e;
      sum += (double)e;
    }
    float inv = (float)(1 / sum);
    for (int i = 0; i < n; i++) o[i] *= inv;
  }
}

/* backend/cpu/cpu.go:53 SiluMul. */
void or_silu_mul(const float *gate, const float *up, float *out, int64_t n) {
  for (int64_t i = 0; i < n; i++) {
    float g = gate[i];
    out[i] = g / (1 + (float)exp((double)(-g))) * up[i];
  }
}

/* backend/cpu/cpu.go:60 Add. */
void or_add(const float *a, const float *b, float *out, int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

/* backend/cpu/cpu.go:69 RoPE (interleaved pairs). */
void or_rope(float *x, const int32_t *pos, const float *freq, int rows, int n_heads,
             int head_dim, float base) {
  for (int r = 0; r < rows; r++) {
    double p = (double)pos[r];
    for (int h = 0; h < n_heads; h++) {
      float *row = x + ((int64_t)r * n_heads + h) * head_dim;
      for (int j = 0; j < head_dim / 2; j++) {
        double theta = p * pow((double)base, -2 * (double)j / (double)head_dim);
        if (freq) theta /= (double)freq[j];
        double s = sin(theta), c = cos(theta);
        double x0 = row[2 * j], x1 = row[2 * j + 1];
        row[2 * j] = (float)(x0 * c - x1 * s);
        row[2 * j + 1] = (float)(x0 * s + x1 * c);
      }
    }
  }
}

/* backend/cpu/cpu.go:90 MatVecF16. */
void or_matvec_f16(const uint16_t *w, const float *x, float *y, int rows, int cols, int batch) {
  for (int b = 0; b < batch; b++)
    for (int r = 0; r < rows; r++) {
      double acc = 0;
      for (int c = 0; c < cols; c++)
        acc += (double)or_f16_to_f32(w[(int64_t)r * cols + c]) * (double)x[(int64_t)b * cols + c];
      y[(int64_t)b * rows + r] = (float)acc;
    }
}

/* backend/cpu/cpu.go:105 MatVecF32. */
void or_matvec_f32(const float *w, const float *x, float *y, int rows, int cols, int batch) {
  for (int b = 0; b < batch; b++)
    for (int r = 0; r < rows; r++) {
      double acc = 0;
      for (int c = 0; c < cols; c++)
        acc += (double)w[(int64_t)r * cols + c] * (double)x[(int64_t)b * cols + c];
      y[(int64_t)b * rows + r] = (float)acc;
    }
}

/* backend/cpu/cpu.go:122 MatVecQ: dequantize each row (quant.Row), then a
 * float64 dot product per batch vector. */
typedef struct {
  int typ; const uint8_t *w; int64_t len; const float *x; float *y;
  int rows, cols, batch, r0, r1, err;
} mv_job;

static void *mv_rows(void *arg) {
  mv_job *j = (mv_job *)arg;
  float *row = (float *)malloc(sizeof(float) * (size_t)j->cols);
  if (!row) { j->err = -4; return NULL; }
  for (int r = j->r0; r < j->r1; r++) {
    int e = or_row(j->typ, j->w, j->len, j->cols, r, row);
    if (e) { j->err = e; break; }
    for (int b = 0; b < j->batch; b++) {
      const float *xb = j->x + (int64_t)b * j->cols;
      double acc = 0;
      for (int c = 0; c < j->cols; c++) acc += (double)row[c] * (double)xb[c];
      j->y[(int64_t)b * j->rows + r] = (float)acc;
    }
  }
  free(row);
  return NULL;
}

int or_matvec_q(int typ, const uint8_t *w, int64_t len, const float *x, float *y, int rows,
                int cols, int batch, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads > rows) threads = rows > 0 ? rows : 1;
  mv_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < threads; t++) {
    mv_job j = {typ, w, len, x, y, rows, cols, batch,
                (int)((int64_t)rows * t / threads), (int)((int64_t)rows * (t + 1) / threads), 0};
    jobs[t] = j;
  }
  if (threads == 1) {
    mv_rows(&jobs[0]);
    return jobs[0].err;
  }
  for (int t = 0; t < threads; t++) pthread_create(&th[t], NULL, mv_rows, &jobs[t]);
  int err = 0;
  for (int t = 0; t < threads; t++) {
    pthread_join(th[t], NULL);
    if (jobs[t].err) err = jobs[t].err;
  }
  return err;
}

/* backend/cpu/cpu.go:143 AttnDecode, heads [h0, h1). */
static void attn_heads(const float *q, const float *kcache, const float *vcache, float *out,
                       int kv_len, int n_heads, int n_kv, int head_dim, float scale, int h0, int h1) {
  int group = n_heads / n_kv, kv_dim = n_kv * head_dim;
  float *scores = (float *)malloc(sizeof(float) * (size_t)(kv_len > 0 ? kv_len : 1));
  for (int h = h0; h < h1; h++) {
    const float *qh = q + (int64_t)h * head_dim;
    int kvh = h / group;
    for (int t = 0; t < kv_len; t++) {
      const float *k = kcache + (int64_t)t * kv_dim + (int64_t)kvh * head_dim;
      double dot = 0;
      for (int d = 0; d < head_dim; d++) dot += (double)qh[d] * (double)k[d];
      scores[t] = (float)dot * scale;
    }
    or_softmax(scores, scores, 1, kv_len);
    float *o = out + (int64_t)h * head_dim;
    for (int d = 0; d < head_dim; d++) {
      double acc = 0;
      for (int t = 0; t < kv_len; t++)
        acc += (double)scores[t] * (double)vcache[(int64_t)t * kv_dim + (int64_t)kvh * head_dim + d];
      o[d] = (float)acc;
    }
  }
  free(scores);
}

void or_attn_decode(const float *q, const float *kcache, const float *vcache, float *out,
                    int kv_len, int n_heads, int n_kv, int head_dim, float scale) {
  attn_heads(q, kcache, vcache, out, kv_len, n_heads, n_kv, head_dim, scale, 0, n_heads);
}

/* Heads are independent, so splitting them across threads changes no bit. */
typedef struct {
  const float *q, *k, *v; float *out;
  int kv_len, n_heads, n_kv, head_dim; float scale; int h0, h1;
} attn_job;

static void *attn_run(void *arg) {
  attn_job *j = (attn_job *)arg;
  attn_heads(j->q, j->k, j->v, j->out, j->kv_len, j->n_heads, j->n_kv, j->head_dim, j->scale,
             j->h0, j->h1);
  return NULL;
}

static void attn_parallel(const float *q, const float *kcache, const float *vcache, float *out,
                          int kv_len, int n_heads, int n_kv, int head_dim, float scale, int threads) {
  if (threads > n_heads) threads = n_heads;
  if (threads > 256) threads = 256;
  if (threads <= 1) {
    or_attn_decode(q, kcache, vcache, out, kv_len, n_heads, n_kv, head_dim, scale);
    return;
  }
  attn_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < threads; t++) {
    attn_job j = {q, kcache, vcache, out, kv_len, n_heads, n_kv, head_dim, scale,
                  n_heads * t / threads, n_heads * (t + 1) / threads};
    jobs[t] = j;
    pthread_create(&th[t], NULL, attn_run, &jobs[t]);
  }
  for (int t = 0; t < threads; t++) pthread_join(th[t], NULL);
}

/* model/model.go:376 Argmax. */
int32_t or_argmax(const float *logits, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 0; i < n; i++)
    if (logits[i] > logits[best]) best = i;
  return (int32_t)best;
}

/* ---- GGUF reader (gguf/gguf.go:62 Parse) -------------------------------- */

enum { VT_U8, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL, VT_STR, VT_ARR,
       VT_U64, VT_I64, VT_F64 };

typedef struct {
  const char *key; uint64_t key_len;
  uint32_t type;
  uint64_t u;      /* integer value as Go's Value.Uint64 */
  double f;        /* float value */
  const char *s; uint64_t s_len;
} or_kv;

typedef struct {
  const char *name; uint64_t name_len;
  uint32_t ndims; uint64_t dims[4];
  uint32_t type; uint64_t offset;
} or_tensor;

struct or_gguf {
  const uint8_t *data; size_t len;
  uint32_t version, alignment;
  or_kv *kv; uint64_t n_kv;
  or_tensor *t; uint64_t n_t;
  uint64_t data_offset;
};

typedef struct { const uint8_t *b; size_t len, pos; const char *err; } rd;

static int need(rd *r, uint64_t n) {
  if (r->err) return 0;
  if (n > r->len || r->pos + n > r->len) { r->err = "gguf: truncated header"; return 0; }
  return 1;
}
static uint64_t rd_le(rd *r, int n) {
  if (!need(r, (uint64_t)n)) return 0;
  uint64_t v = 0;
  for (int i = 0; i < n; i++) v |= (uint64_t)r->b[r->pos + i] << (8 * i);
  r->pos += (size_t)n;
  return v;
}
static const char *rd_str(rd *r, uint64_t *n) {
  *n = rd_le(r, 8);
  if (*n > r->len || !need(r, *n)) {
    if (!r->err) r->err = "gguf: bad string length";
    *n = 0;
    return "";
  }
  const char *s = (const char *)r->b + r->pos;
  r->pos += (size_t)*n;
  return s;
}

/* gguf/gguf.go:391 typed. Scalars are decoded into kv; arrays are walked. */
static int rd_typed(rd *r, uint32_t t, or_kv *kv, int depth) {
  uint64_t v;
  if (kv) { kv->type = t; kv->u = 0; kv->f = 0; }
  switch (t) {
    case VT_U8: v = rd_le(r, 1); if (kv) kv->u = v; break;
    case VT_I8: v = rd_le(r, 1); if (kv) kv->u = (uint64_t)(int64_t)(int8_t)v; break;
    case VT_U16: v = rd_le(r, 2); if (kv) kv->u = v; break;
    case VT_I16: v = rd_le(r, 2); if (kv) kv->u = (uint64_t)(int64_t)(int16_t)v; break;
    case VT_U32: v = rd_le(r, 4); if (kv) kv->u = v; break;
    case VT_I32: v = rd_le(r, 4); if (kv) kv->u = (uint64_t)(int64_t)(int32_t)v; break;
    case VT_F32: v = rd_le(r, 4); if (kv) kv->f = f32_from_bits((uint32_t)v); break;
    case VT_BOOL: v = rd_le(r, 1); if (kv) kv->u = v != 0; break;
    case VT_STR: { uint64_t n; const char *s = rd_str(r, &n); if (kv) { kv->s = s; kv->s_len = n; } break; }
    case VT_U64: v = rd_le(r, 8); if (kv) kv->u = v; break;
    case VT_I64: v = rd_le(r, 8); if (kv) kv->u = v; break;
    case VT_F64: v = rd_le(r, 8); if (kv) { double d; memcpy(&d, &v, 8); kv->f = d; } break;
    case VT_ARR: {
      uint32_t elem = (uint32_t)rd_le(r, 4);
      uint64_t n = rd_le(r, 8);
      if (n > r->len) { r->err = "gguf: bad array length"; return -1; }
      if (depth > 16) { r->err = "gguf: arrays nested too deep"; return -1; }
      for (uint64_t i = 0; i < n && !r->err; i++)
        if (rd_typed(r, elem, NULL, depth + 1)) return -1;
      break;
    }
    default: r->err = "gguf: unknown value type"; return -1;
  }
  return r->err ? -1 : 0;
}

static int key_eq(const char *a, uint64_t alen, const char *b) {
  return strlen(b) == alen && memcmp(a, b, alen) == 0;
}

or_gguf *or_gguf_parse(const uint8_t *data, size_t len, char *err, int errlen) {
  rd r = {data, len, 0, NULL};
  or_gguf *f = (or_gguf *)calloc(1, sizeof(or_gguf));
  const char *msg = NULL;
  f->data = data; f->len = len; f->alignment = 32;
  if (rd_le(&r, 4) != 0x46554747u) { msg = "gguf: bad magic"; goto fail; }
  f->version = (uint32_t)rd_le(&r, 4);
  if (r.err) { msg = r.err; goto fail; }
  if (f->version < 2 || f->version > 3) { msg = "gguf: unsupported version"; goto fail; }
  uint64_t n_t = rd_le(&r, 8), n_kv = rd_le(&r, 8);
  if (r.err) { msg = r.err; goto fail; }
  if (n_kv > len || n_t > len) { msg = "gguf: corrupt header counts"; goto fail; }
  f->kv = (or_kv *)calloc(n_kv ? n_kv : 1, sizeof(or_kv));
  for (uint64_t i = 0; i < n_kv; i++) {
    or_kv *kv = &f->kv[i];
    kv->key = rd_str(&r, &kv->key_len);
    uint32_t t = (uint32_t)rd_le(&r, 4);
    if (r.err || rd_typed(&r, t, kv, 0)) { msg = r.err ? r.err : "gguf: bad value"; goto fail; }
    f->n_kv = i + 1;
    if (key_eq(kv->key, kv->key_len, "general.alignment")) {
      uint64_t a = (kv->type == VT_F32 || kv->type == VT_F64 || kv->type == VT_STR) ? 0 : kv->u;
      f->alignment = (uint32_t)a;
    }
  }
  if (f->alignment == 0 || (f->alignment & (f->alignment - 1)) != 0) {
    msg = "gguf: bad alignment"; goto fail;
  }
  f->t = (or_tensor *)calloc(n_t ? n_t : 1, sizeof(or_tensor));
  for (uint64_t i = 0; i < n_t; i++) {
    or_tensor *t = &f->t[i];
    t->name = rd_str(&r, &t->name_len);
    t->ndims = (uint32_t)rd_le(&r, 4);
    if (r.err) { msg = r.err; goto fail; }
    if (t->ndims > 4) { msg = "gguf: tensor has more than 4 dims"; goto fail; }
    for (uint32_t j = 0; j < t->ndims; j++) t->dims[j] = rd_le(&r, 8);
    t->type = (uint32_t)rd_le(&r, 4);
    t->offset = rd_le(&r, 8);
    if (r.err) { msg = r.err; goto fail; }
    if (or_block_size((int)t->type) == 0) { msg = "gguf: unknown tensor type"; goto fail; }
    for (uint64_t k = 0; k < i; k++)
      if (f->t[k].name_len == t->name_len && memcmp(f->t[k].name, t->name, t->name_len) == 0) {
        msg = "gguf: duplicate tensor"; goto fail;
      }
    f->n_t = i + 1;
  }
  f->data_offset = (r.pos + f->alignment - 1) & ~(uint64_t)(f->alignment - 1);
  for (uint64_t i = 0; i < f->n_t; i++) {
    or_tensor *t = &f->t[i];
    uint64_t bytes = 0;
    if (t->ndims) {
      uint64_t ne = 1;
      for (uint32_t j = 0; j < t->ndims; j++) ne *= t->dims[j];
      bytes = t->dims[0] ? (uint64_t)or_row_bytes((int)t->type, (int64_t)t->dims[0]) * (ne / t->dims[0]) : 0;
    }
    uint64_t end = f->data_offset + t->offset + bytes;
    if (t->offset % f->alignment != 0 || end > len) { msg = "gguf: tensor data out of range"; goto fail; }
  }
  return f;
fail:
  if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", msg ? msg : "gguf: parse error");
  or_gguf_free(f);
  return NULL;
}

void or_gguf_free(or_gguf *f) {
  if (!f) return;
  free(f->kv);
  free(f->t);
  free(f);
}

uint32_t or_gguf_version(const or_gguf *f) { return f->version; }
uint32_t or_gguf_alignment(const or_gguf *f) { return f->alignment; }
int or_gguf_n_tensors(const or_gguf *f) { return (int)f->n_t; }
int or_gguf_n_kv(const or_gguf *f) { return (int)f->n_kv; }

static const or_kv *find_kv(const or_gguf *f, const char *key) {
  for (uint64_t i = 0; i < f->n_kv; i++)
    if (key_eq(f->kv[i].key, f->kv[i].key_len, key)) return &f->kv[i];
  return NULL;
}

/* gguf/gguf.go:155 Uint: any integer type, else def. */
uint64_t or_gguf_uint(const or_gguf *f, const char *key, uint64_t def) {
  const or_kv *kv = find_kv(f, key);
  if (!kv) return def;
  switch (kv->type) {
    case VT_U8: case VT_I8: case VT_U16: case VT_I16: case VT_U32: case VT_I32:
    case VT_U64: case VT_I64: return kv->u;
  }
  return def;
}

/* gguf/gguf.go:163 Float: float32 or float64 only. */
double or_gguf_float(const or_gguf *f, const char *key, double def) {
  const or_kv *kv = find_kv(f, key);
  if (kv && (kv->type == VT_F32 || kv->type == VT_F64)) return kv->f;
  return def;
}

void or_gguf_string(const or_gguf *f, const char *key, const char *def, char *out, int cap) {
  const or_kv *kv = find_kv(f, key);
  if (cap <= 0) return;
  if (kv && kv->type == VT_STR) {
    uint64_t n = kv->s_len < (uint64_t)(cap - 1) ? kv->s_len : (uint64_t)(cap - 1);
    memcpy(out, kv->s, n);
    out[n] = 0;
  } else {
    snprintf(out, (size_t)cap, "%s", def ? def : "");
  }
}

int or_gguf_tensor(const or_gguf *f, const char *name, int *type, int *ndims, uint64_t *dims,
                   const uint8_t **data, uint64_t *nbytes) {
  for (uint64_t i = 0; i < f->n_t; i++) {
    const or_tensor *t = &f->t[i];
    if (!key_eq(t->name, t->name_len, name)) continue;
    uint64_t ne = 1;
    for (uint32_t j = 0; j < t->ndims; j++) ne *= t->dims[j];
    if (type) *type = (int)t->type;
    if (ndims) *ndims = (int)t->ndims;
    if (dims) for (uint32_t j = 0; j < t->ndims; j++) dims[j] = t->dims[j];
    uint64_t bytes = t->ndims && t->dims[0]
        ? (uint64_t)or_row_bytes((int)t->type, (int64_t)t->dims[0]) * (ne / t->dims[0]) : 0;
    if (data) *data = f->data + f->data_offset + t->offset;
    if (nbytes) *nbytes = bytes;
    return 0;
  }
  return -1;
}

/* ---- cpuForward (model/model_test.go:114-175) --------------------------- */

typedef struct { int type; int rows, cols; const uint8_t *data; uint64_t bytes; } or_mat;

struct or_model {
  or_gguf *f;
  or_config c;
  int max_len, kv_f16;
  or_mat embd, head;
  float **kc, **vc;          /* [layer][max_len * kv_dim] */
  float *freq;               /* NULL when the file has no rope_freqs.weight */
};

static int get_mat(or_gguf *f, const char *name, or_mat *m) {
  int nd; uint64_t dims[4];
  if (or_gguf_tensor(f, name, &m->type, &nd, dims, &m->data, &m->bytes)) return -1;
  if (nd == 1) { m->rows = 1; m->cols = (int)dims[0]; }
  else if (nd == 2) { m->rows = (int)dims[1]; m->cols = (int)dims[0]; }
  else return -2;
  return 0;
}

/* cpuForward's vec(): the whole tensor dequantized. */
static float *vec(or_gguf *f, const char *name, int n) {
  or_mat m;
  if (get_mat(f, name, &m)) return NULL;
  if ((int64_t)m.rows * m.cols != n) return NULL;
  float *out = (float *)malloc(sizeof(float) * (size_t)n);
  if (or_dequantize(m.type, m.data, (int64_t)m.bytes, out, n)) { free(out); return NULL; }
  return out;
}

or_model *or_model_open(const uint8_t *gguf, size_t len, int max_len, int kv_f16, char *err,
                        int errlen) {
  or_gguf *f = or_gguf_parse(gguf, len, err, errlen);
  if (!f) return NULL;
  char arch[64];
  or_gguf_string(f, "general.architecture", "", arch, sizeof arch);
  if (strcmp(arch, "llama") != 0) {
    snprintf(err, (size_t)errlen, "model: architecture %s is not llama", arch);
    or_gguf_free(f);
    return NULL;
  }
  /* model/model.go:35 ConfigFrom */
  or_config c;
  c.layers = (int)or_gguf_uint(f, "llama.block_count", 0);
  c.dim = (int)or_gguf_uint(f, "llama.embedding_length", 0);
  c.ffn = (int)or_gguf_uint(f, "llama.feed_forward_length", 0);
  c.heads = (int)or_gguf_uint(f, "llama.attention.head_count", 0);
  c.ctx_len = (int)or_gguf_uint(f, "llama.context_length", 2048);
  c.rope_base = (float)or_gguf_float(f, "llama.rope.freq_base", 10000);
  c.eps = (float)or_gguf_float(f, "llama.attention.layer_norm_rms_epsilon", 1e-5);
  c.kv_heads = (int)or_gguf_uint(f, "llama.attention.head_count_kv", (uint64_t)c.heads);
  if (!c.layers || !c.dim || !c.ffn || !c.heads || !c.kv_heads) {
    snprintf(err, (size_t)errlen, "model: incomplete llama metadata");
    or_gguf_free(f);
    return NULL;
  }
  c.head_dim = (int)or_gguf_uint(f, "llama.attention.key_length", (uint64_t)(c.dim / c.heads));
  or_model *m = (or_model *)calloc(1, sizeof(or_model));
  m->f = f;
  if (get_mat(f, "token_embd.weight", &m->embd)) {
    snprintf(err, (size_t)errlen, "model: no token_embd.weight");
    or_model_free(m);
    return NULL;
  }
  c.vocab = m->embd.rows;
  if (get_mat(f, "output.weight", &m->head)) m->head = m->embd; /* tied */
  if (max_len <= 0 || max_len > c.ctx_len) max_len = c.ctx_len;
  m->c = c;
  m->max_len = max_len;
  m->kv_f16 = kv_f16;
  int kv_dim = c.kv_heads * c.head_dim;
  m->kc = (float **)calloc((size_t)c.layers, sizeof(float *));
  m->vc = (float **)calloc((size_t)c.layers, sizeof(float *));
  for (int i = 0; i < c.layers; i++) {
    m->kc[i] = (float *)calloc((size_t)max_len * kv_dim, sizeof(float));
    m->vc[i] = (float *)calloc((size_t)max_len * kv_dim, sizeof(float));
    if (!m->kc[i] || !m->vc[i]) {
      snprintf(err, (size_t)errlen, "model: out of host memory for the KV cache");
      or_model_free(m);
      return NULL;
    }
  }
  int nd; uint64_t dims[4];
  if (or_gguf_tensor(f, "rope_freqs.weight", NULL, &nd, dims, NULL, NULL) == 0)
    m->freq = vec(f, "rope_freqs.weight", c.head_dim / 2);
  return m;
}

void or_model_free(or_model *m) {
  if (!m) return;
  if (m->kc) for (int i = 0; i < m->c.layers; i++) free(m->kc[i]);
  if (m->vc) for (int i = 0; i < m->c.layers; i++) free(m->vc[i]);
  free(m->kc);
  free(m->vc);
  free(m->freq);
  or_gguf_free(m->f);
  free(m);
}

void or_model_config(const or_model *m, or_config *c) { *c = m->c; }
const float *or_model_kcache(const or_model *m, int layer) { return m->kc[layer]; }
const float *or_model_vcache(const or_model *m, int layer) { return m->vc[layer]; }

int or_model_set_kv(or_model *m, int layer, int pos0, int n, const float *k, const float *v) {
  int kv_dim = m->c.kv_heads * m->c.head_dim;
  if (layer < 0 || layer >= m->c.layers || pos0 < 0 || n < 0 || pos0 + n > m->max_len) return -1;
  memcpy(m->kc[layer] + (int64_t)pos0 * kv_dim, k, sizeof(float) * (size_t)n * kv_dim);
  memcpy(m->vc[layer] + (int64_t)pos0 * kv_dim, v, sizeof(float) * (size_t)n * kv_dim);
  return 0;
}

/* cpuForward's matvec(): cpu.MatVecQ for quantized weights, MatVecF32/F16
 * otherwise (the reference only feeds quantized matrices to it). */
static int matvec(or_gguf *f, const char *name, const float *x, float *y, int rows, int cols,
                  int threads) {
  or_mat m;
  if (get_mat(f, name, &m) || m.rows != rows || m.cols != cols) return -1;
  return or_matvec_q(m.type, m.data, (int64_t)m.bytes, x, y, rows, cols, 1, threads);
}

int or_model_forward(or_model *m, int32_t token, int pos, float *logits, int threads) {
  const or_config c = m->c;
  or_gguf *f = m->f;
  if (pos < 0 || pos >= m->max_len || token < 0 || token >= c.vocab) return -1;
  int kv_dim = c.kv_heads * c.head_dim, qdim = c.heads * c.head_dim;
  float *x = (float *)malloc(sizeof(float) * (size_t)c.dim);
  float *xn = (float *)malloc(sizeof(float) * (size_t)c.dim);
  float *q = (float *)malloc(sizeof(float) * (size_t)qdim);
  float *k = (float *)malloc(sizeof(float) * (size_t)kv_dim);
  float *v = (float *)malloc(sizeof(float) * (size_t)kv_dim);
  float *attn = (float *)malloc(sizeof(float) * (size_t)qdim);
  float *o = (float *)malloc(sizeof(float) * (size_t)c.dim);
  float *gate = (float *)malloc(sizeof(float) * (size_t)c.ffn);
  float *up = (float *)malloc(sizeof(float) * (size_t)c.ffn);
  int rc = 0;
  int32_t posv = pos;
  float scale = (float)(1 / sqrt((double)c.head_dim));
  char name[96];
  if (or_row(m->embd.type, m->embd.data, (int64_t)m->embd.bytes, c.dim, token, x)) { rc = -2; goto done; }
  for (int i = 0; i < c.layers && rc == 0; i++) {
    snprintf(name, sizeof name, "blk.%d.attn_norm.weight", i);
    float *an = vec(f, name, c.dim);
    if (!an) { rc = -3; break; }
    or_rmsnorm(x, an, xn, 1, c.dim, c.eps);
    free(an);
    snprintf(name, sizeof name, "blk.%d.attn_q.weight", i);
    rc |= matvec(f, name, xn, q, qdim, c.dim, threads);
    snprintf(name, sizeof name, "blk.%d.attn_k.weight", i);
    rc |= matvec(f, name, xn, k, kv_dim, c.dim, threads);
    snprintf(name, sizeof name, "blk.%d.attn_v.weight", i);
    rc |= matvec(f, name, xn, v, kv_dim, c.dim, threads);
    if (rc) break;
    or_rope(q, &posv, m->freq, 1, c.heads, c.head_dim, c.rope_base);
    or_rope(k, &posv, m->freq, 1, c.kv_heads, c.head_dim, c.rope_base);
    float *kr = m->kc[i] + (int64_t)pos * kv_dim, *vr = m->vc[i] + (int64_t)pos * kv_dim;
    for (int j = 0; j < kv_dim; j++) {
      kr[j] = m->kv_f16 ? or_f16_to_f32(or_f16_from(k[j])) : k[j];
      vr[j] = m->kv_f16 ? or_f16_to_f32(or_f16_from(v[j])) : v[j];
    }
    attn_parallel(q, m->kc[i], m->vc[i], attn, pos + 1, c.heads, c.kv_heads, c.head_dim, scale,
                  threads);
    snprintf(name, sizeof name, "blk.%d.attn_output.weight", i);
    rc |= matvec(f, name, attn, o, c.dim, qdim, threads);
    if (rc) break;
    or_add(x, o, x, c.dim);
    snprintf(name, sizeof name, "blk.%d.ffn_norm.weight", i);
    float *fn = vec(f, name, c.dim);
    if (!fn) { rc = -3; break; }
    or_rmsnorm(x, fn, xn, 1, c.dim, c.eps);
    free(fn);
    snprintf(name, sizeof name, "blk.%d.ffn_gate.weight", i);
    rc |= matvec(f, name, xn, gate, c.ffn, c.dim, threads);
    snprintf(name, sizeof name, "blk.%d.ffn_up.weight", i);
    rc |= matvec(f, name, xn, up, c.ffn, c.dim, threads);
    if (rc) break;
    or_silu_mul(gate, up, gate, c.ffn);
    snprintf(name, sizeof name, "blk.%d.ffn_down.weight", i);
    rc |= matvec(f, name, gate, o, c.dim, c.ffn, threads);
    if (rc) break;
    or_add(x, o, x, c.dim);
  }
  if (rc == 0) {
    float *on = vec(f, "output_norm.weight", c.dim);
    if (!on) rc = -3;
    else {
      or_rmsnorm(x, on, xn, 1, c.dim, c.eps);
      free(on);
      rc = or_matvec_q(m->head.type, m->head.data, (int64_t)m->head.bytes, xn, logits, c.vocab,
                       c.dim, 1, threads);
    }
  }
done:
  free(x); free(xn); free(q); free(k); free(v); free(attn); free(o); free(gate); free(up);
  return rc;
}

/* ---- sampler (the B200 build's rule, restated; see oracle.h) -------------- */

enum { SMP_T = 1024, SMP_MAXK = 1024 };

float or_exp_nonpos(float x) {
  if (!(x >= -87.f)) return 0.f;
  float n = rintf(x * 1.44269502f);
  float r = fmaf(-n, 0.693359375f, x);
  r = fmaf(-n, -2.12194440e-4f, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333333e-3f);
  p = fmaf(p, r, 4.16666667e-2f);
  p = fmaf(p, r, 1.66666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.f);
  p = fmaf(p, r, 1.f);
  uint32_t b = (uint32_t)((int)n + 127) << 23;
  float s;
  memcpy(&s, &b, 4);
  return p * s;
}

float or_uniform24(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1ull) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(uint32_t)(z >> 40) * (1.f / 16777216.f);
}

static uint32_t smp_okey(float f) {
  if (f != f) return 0u;
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b << 1) == 0u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
static float smp_okey_value(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static void smp_scan(float *a) { /* Hillis-Steele, a[i] = a[i-d] + a[i] */
  static __thread float nb[SMP_T];
  for (int d = 1; d < SMP_T; d <<= 1) {
    for (int i = 0; i < SMP_T; i++) nb[i] = i >= d ? a[i - d] + a[i] : a[i];
    memcpy(a, nb, sizeof nb);
  }
}

static int smp_desc(const void *x, const void *y) {
  uint64_t a = *(const uint64_t *)x, b = *(const uint64_t *)y;
  return a < b ? 1 : a > b ? -1 : 0;
}

int32_t or_sample(const float *logits, int n, const or_sample_params *p, const int32_t *recent,
                  int n_recent, uint64_t counter) {
  if (n <= 0) return 0;
  uint8_t *pen = NULL;
  if (p->repeat_penalty != 1.f && p->repeat_last_n > 0) {
    pen = calloc((size_t)n, 1);
    int lo = n_recent - p->repeat_last_n;
    for (int q = lo < 0 ? 0 : lo; q < n_recent; q++)
      if (recent[q] >= 0 && recent[q] < n) pen[recent[q]] = 1;
  }
  const int greedy = !(p->temperature > 0.f) || p->top_k == 1;
  const float t = greedy ? 0.f : p->temperature, rp = p->repeat_penalty;
  float *s = malloc(sizeof(float) * (size_t)n);
  for (int i = 0; i < n; i++) {
    float v = logits[i];
    if (pen && pen[i]) v = v <= 0.f ? v * rp : v / rp;
    if (t > 0.f) v = v / t;
    s[i] = v;
  }
  free(pen);
  uint64_t best = 0;
  for (int i = 0; i < n; i++) {
    uint64_t k = ((uint64_t)smp_okey(s[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    if (k > best) best = k;
  }
  const int arg = (int)(0xFFFFFFFFu - (uint32_t)best);
  const float mx = smp_okey_value((uint32_t)(best >> 32));
  int pick = arg;
  const float u = or_uniform24(p->seed, counter);
  if (greedy) {
  } else if (p->top_k <= 0 && !(p->top_p < 1.f)) {
    const int C = (n + SMP_T - 1) / SMP_T;
    float cum[SMP_T];
    for (int th = 0; th < SMP_T; th++) {
      int c0 = th * C < n ? th * C : n, c1 = c0 + C < n ? c0 + C : n;
      float local = 0.f;
      for (int i = c0; i < c1; i++) local = local + or_exp_nonpos(s[i] - mx);
      cum[th] = local;
    }
    smp_scan(cum);
    const float target = u * cum[SMP_T - 1];
    for (int th = 0; th < SMP_T; th++) {
      int c0 = th * C < n ? th * C : n, c1 = c0 + C < n ? c0 + C : n, hit = -1;
      float acc = th ? cum[th - 1] : 0.f;
      for (int i = c0; i < c1; i++) {
        acc = acc + or_exp_nonpos(s[i] - mx);
        if (acc > target) {
          hit = i;
          break;
        }
      }
      if (hit >= 0) {
        pick = hit;
        break;
      }
    }
  } else {
    int K = (p->top_k <= 0 || p->top_k > SMP_MAXK) ? SMP_MAXK : p->top_k;
    if (K > n) K = n;
    uint64_t *keys = malloc(sizeof(uint64_t) * (size_t)n);
    for (int i = 0; i < n; i++) keys[i] = ((uint64_t)smp_okey(s[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    qsort(keys, (size_t)n, sizeof(uint64_t), smp_desc);
    float cum[SMP_T];
    const float v0 = smp_okey_value((uint32_t)(keys[0] >> 32));
    for (int i = 0; i < SMP_T; i++) cum[i] = i < K ? or_exp_nonpos(smp_okey_value((uint32_t)(keys[i] >> 32)) - v0) : 0.f;
    smp_scan(cum);
    int c = K - 1;
    if (p->top_p < 1.f) {
      const float thr = p->top_p * cum[SMP_T - 1];
      for (int i = 0; i < SMP_T; i++)
        if (cum[i] >= thr) {
          c = i;
          break;
        }
      if (c > K - 1) c = K - 1;
    }
    const float target = u * cum[c];
    int slot = 0;
    for (int i = 0; i <= c; i++)
      if (cum[i] > target) {
        slot = i;
        break;
      }
    pick = (int)(0xFFFFFFFFu - (uint32_t)keys[slot]);
    free(keys);
  }
  free(s);
  return pick;
}
