/*
 * oracle.h -- CPU restatement of gollama.cu's pure-Go reference path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the
 * B200 decode path: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load it. The product library
 * (gollama.cu_b200/) never links, loads or calls it.
 *
 * Every function restates one Go function of the reference, cited by
 * file:line inside the reference project. Go is not available on this
 * machine, so the Go sources cannot be built; the restatement is pinned
 * against the known-answer vectors of the reference's own tests
 * (quant/quant_test.go, f16/f16_test.go, gguf/gguf_test.go) and against
 * hand-derived Q4_K / Q6_K blocks (tests/golden/).
 *
 * Floating point follows Go on amd64: float32 operations round to float32
 * individually (built with -ffp-contract=off), float64 accumulators where
 * the Go code uses them.
 */
#ifndef GOLLAMA_ORACLE_H
#define GOLLAMA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (gguf/types.go:8-37). */
enum {
  OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q4_K = 12,
  OR_Q5_K = 13, OR_Q6_K = 14, OR_BF16 = 30
};

/* gguf/types.go:47-57 block size / type size; 0 when unknown. */
int or_block_size(int typ);
int or_type_size(int typ);
/* gguf/types.go:81 RowBytes. */
int64_t or_row_bytes(int typ, int64_t n);

/* f16/f16.go:11 From (round to nearest even) and :47 Float32. */
uint16_t or_f16_from(float x);
float or_f16_to_f32(uint16_t h);

/* quant/quant.go:27 Dequantize: decode n elements of typ. Returns 0, or
 * -1 (n not a block multiple), -2 (data too short), -3 (unsupported). */
int or_dequantize(int typ, const uint8_t *data, int64_t len, float *out, int64_t n);
/* quant/quant.go:135 Row. */
int or_row(int typ, const uint8_t *data, int64_t len, int cols, int64_t r, float *out);
/* quant/quant.go:90 ScaleMinQ4K. */
void or_scale_min_q4k(const uint8_t *scales, int j, uint8_t *sc, uint8_t *m);

/* backend/cpu/cpu.go twins. */
void or_rmsnorm(const float *x, const float *w, float *out, int rows, int n, float eps);
void or_softmax(const float *x, float *out, int rows, int n);
void or_silu_mul(const float *gate, const float *up, float *out, int64_t n);
void or_add(const float *a, const float *b, float *out, int64_t n);
void or_rope(float *x, const int32_t *pos, const float *freq, int rows, int n_heads,
             int head_dim, float base);
void or_matvec_f16(const uint16_t *w, const float *x, float *y, int rows, int cols, int batch);
void or_matvec_f32(const float *w, const float *x, float *y, int rows, int cols, int batch);
/* cpu.MatVecQ; rows are independent, so `threads` > 1 splits rows across
 * threads without changing a single bit of the result. */
int or_matvec_q(int typ, const uint8_t *w, int64_t len, const float *x, float *y, int rows,
                int cols, int batch, int threads);
void or_attn_decode(const float *q, const float *kcache, const float *vcache, float *out,
                    int kv_len, int n_heads, int n_kv, int head_dim, float scale);

/* model/model.go:376 Argmax (first maximum wins; NaN never wins). */
int32_t or_argmax(const float *logits, int64_t n);

/* ---- GGUF reader (gguf/gguf.go:62 Parse) -------------------------------- */
typedef struct or_gguf or_gguf;
/* Parses a GGUF image held in memory (not copied; must outlive the handle).
 * Returns NULL and writes a message into err on failure. */
or_gguf *or_gguf_parse(const uint8_t *data, size_t len, char *err, int errlen);
void or_gguf_free(or_gguf *f);
uint32_t or_gguf_version(const or_gguf *f);
uint32_t or_gguf_alignment(const or_gguf *f);
int or_gguf_n_tensors(const or_gguf *f);
int or_gguf_n_kv(const or_gguf *f);
/* f.Uint / f.Float / f.String with defaults (gguf/gguf.go:155-178). */
uint64_t or_gguf_uint(const or_gguf *f, const char *key, uint64_t def);
double or_gguf_float(const or_gguf *f, const char *key, double def);
/* Copies the string (NUL-terminated, truncated to cap) or def. */
void or_gguf_string(const or_gguf *f, const char *key, const char *def, char *out, int cap);
/* Tensor lookup: returns 0 if found; fills type, ndims, dims (ggml order,
 * innermost first), data pointer and byte size. */
int or_gguf_tensor(const or_gguf *f, const char *name, int *type, int *ndims, uint64_t *dims,
                   const uint8_t **data, uint64_t *nbytes);

/* ---- cpuForward (model/model_test.go:114-175) ---------------------------- */
typedef struct {
  int layers, dim, ffn, heads, kv_heads, head_dim, vocab, ctx_len;
  float rope_base, eps;
} or_config;

typedef struct or_model or_model;
/* model/model.go:35 ConfigFrom + a KV cache of max_len positions.
 * kv_f16 != 0 rounds every stored K/V value through binary16 (f16.From then
 * Float32): the fp16-KV configurations of the B200 build; 0 keeps the
 * reference's float32 cache. Returns NULL with a message on error. */
or_model *or_model_open(const uint8_t *gguf, size_t len, int max_len, int kv_f16, char *err,
                        int errlen);
void or_model_free(or_model *m);
void or_model_config(const or_model *m, or_config *c);
/* One decode step: logits (vocab floats) of token at pos. */
int or_model_forward(or_model *m, int32_t token, int pos, float *logits, int threads);
/* Overwrite cache rows [pos0, pos0+n) of layer with the given float values
 * (already rounded by the caller where the cache is fp16). */
int or_model_set_kv(or_model *m, int layer, int pos0, int n, const float *k, const float *v);
/* Pointer to the cache of one layer ([max_len][kv_dim]), for tests. */
const float *or_model_kcache(const or_model *m, int layer);
const float *or_model_vcache(const or_model *m, int layer);

/* ---- sampler ---------------------------------------------------------------
 * The reference has no sampler (it picks with model.Argmax; sampling is its
 * roadmap item ROADMAP.md:42-45), so this restates the B200 build's own
 * sampling rule (temperature, top-k, top-p, repetition penalty, seeded
 * draw) operation for operation: float32 operations rounded one at a time,
 * fmaf where the rule fuses, and every sum in the rule's fixed association.
 * It is the checker of the device sampler, token for token. */
typedef struct {
  float temperature;
  int top_k;
  float top_p;
  float repeat_penalty;
  int repeat_last_n;
  int reserved;
  uint64_t seed;
} or_sample_params;

/* e^x for x <= 0 by the rule's own method (0 below -87 and for NaN). */
float or_exp_nonpos(float x);
/* The draw in [0, 1): splitmix64 of (seed, counter), 24 bits. */
float or_uniform24(uint64_t seed, uint64_t counter);
/* One token from logits[n]; recent[n_recent] = context ids, oldest first. */
int32_t or_sample(const float *logits, int n, const or_sample_params *p, const int32_t *recent,
                  int n_recent, uint64_t counter);

/* ---- synthetic inputs (synth.c) -------------------------------------------
 * The benchmark's seeded GGUF models and KV prefill, built without the
 * product library (the same bytes as its generator; tests/test_oracle_synth.py). */
typedef struct {
  int layers, dim, ffn, heads, kv_heads, head_dim, vocab, ctx_len;
  float rope_base, eps;
  int mix; /* 0 Q4_0 tied head; 1 Q4_K_M; 2 Q4_K; 3 Q6_K; 4 Q8_0; 5 F16; 6 Q5_K_M */
  uint64_t seed;
} or_synth_spec;
/* Presets 1 (1B Q4_0), 3 (3B Q4_K_M), 8 (8B Q4_K_M), 70 (70B Q4_K_M). */
int or_synth_preset(int preset, or_synth_spec *s);
/* The GGUF image in host memory (or_synth_free). 0 on success. */
int or_synth_model(const or_synth_spec *s, uint8_t **img, size_t *len);
void or_synth_free(uint8_t *img);
/* N(0,1) K and V rows [n][kv_dim] of one layer for positions [pos0, pos0+n),
 * rounded through binary16 when f16 != 0. */
int or_synth_kv_normal(uint64_t seed, int layer, int pos0, int n, int kv_dim, int f16, float *k, float *v);

#ifdef __cplusplus
}
#endif
#endif
