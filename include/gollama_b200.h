/*
 * gollama_b200.h -- C ABI of the B200-native decode path of gollama.cu.
 *
 * This is the drop-in boundary: every entry point takes plain pointers,
 * sizes and scalars (no C++ or torch types) and returns an int status
 * (GB_OK == 0). On failure gb_last_error() returns the message of the
 * calling thread's last failing call, worded like the reference's Go
 * errors ("gpu: <kernel>: ...", "model: ...").
 *
 * Each declaration names the reference interface it replaces, as
 * file:line in the mehdi-shokohi/gollama.cu project. Device pointers are
 * CUDA device addresses on the current device; `stream` is a cudaStream_t
 * (NULL = the legacy default stream, as the reference's nil *cuda.Stream).
 * The caller owns every buffer it passes; handles returned by the library
 * are released with the matching *_close / *_free call.
 */
#ifndef GOLLAMA_B200_H
#define GOLLAMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------ */
#define GB_OK 0
#define GB_ERR_INVALID 1     /* argument rejected (reference: a returned error) */
#define GB_ERR_CUDA 2        /* CUDA runtime error */
#define GB_ERR_UNSUPPORTED 3 /* type or shape without a kernel */
#define GB_ERR_IO 4          /* file or GGUF format error */
#define GB_ERR_NCCL 5        /* NCCL error */
#define GB_ERR_TIMEOUT 6     /* a bounded device wait ran out */
#define GB_ERR_DEVICE 7      /* a kernel reported an error flag */

/* ggml type ids, gguf/types.go:8-37. */
#define GB_F32 0
#define GB_F16 1
#define GB_Q4_0 2
#define GB_Q8_0 8
#define GB_Q4_K 12
#define GB_Q6_K 14
#define GB_BF16 30

/* Message of this thread's last failed call ("" if none). */
const char *gb_last_error(void);
/* Library version string. */
const char *gb_version(void);

/* ---- backend/gpu: the per-kernel launch API ----------------------------- */
typedef struct gb_kernels gb_kernels;

/* gpu.Load, backend/gpu/gpu.go:35. Binds the sm_100a kernels on `device`
 * (the reference loads kernels.ptx into a context). */
int gb_gpu_load(int device, gb_kernels **out);
/* (*Kernels).Len, backend/gpu/gpu.go:53: number of kernels bound. */
int gb_gpu_len(const gb_kernels *k);
/* (*Kernels).Close, backend/gpu/gpu.go:56. */
int gb_gpu_close(gb_kernels *k);

/* (*Kernels).RMSNorm, backend/gpu/gpu.go:91. x and out may alias. */
int gb_gpu_rmsnorm(gb_kernels *k, void *stream, const float *x, const float *w, float *out,
                   int rows, int n, float eps);
/* (*Kernels).Softmax, backend/gpu/gpu.go:96. x and out may alias. */
int gb_gpu_softmax(gb_kernels *k, void *stream, const float *x, float *out, int rows, int n);
/* (*Kernels).SiluMul, backend/gpu/gpu.go:101. */
int gb_gpu_silu_mul(gb_kernels *k, void *stream, const float *gate, const float *up, float *out,
                    int n);
/* (*Kernels).Add, backend/gpu/gpu.go:106. */
int gb_gpu_add(gb_kernels *k, void *stream, const float *a, const float *b, float *out, int n);
/* (*Kernels).RoPE, backend/gpu/gpu.go:112: in place, pos[rows] on the
 * device, freq[head_dim/2] (ones when the model has none). */
int gb_gpu_rope(gb_kernels *k, void *stream, float *x, const int32_t *pos, const float *freq,
                int rows, int n_heads, int head_dim, float base);
/* (*Kernels).AttnDecode, backend/gpu/gpu.go:118: q[n_heads*head_dim],
 * kcache/vcache [kv_len][n_kv*head_dim] float32, out[n_heads*head_dim].
 * Split-K flash decode; its partial results live in a workspace owned by
 * `k` (allocated on first use, grown when a larger kv_len needs more). */
int gb_gpu_attn_decode(gb_kernels *k, void *stream, const float *q, const float *kcache,
                       const float *vcache, float *out, int kv_len, int n_heads, int n_kv,
                       int head_dim, float scale);
/* AttnDecode with no allocation: no counterpart in the reference. The same
 * arguments and results as gb_gpu_attn_decode, but the slice partials and
 * counters live in fixed device arrays of this library (at most 2^20 floats
 * of partials, i.e. n_kv * slices * (n_heads/n_kv) * (head_dim + 4), and at
 * most 256 KV heads); larger requests fail with GB_ERR_UNSUPPORTED and a
 * message naming the limit. It calls no cudaMalloc or cudaFree. The first
 * call on a device resolves the arrays' addresses for that device, so make
 * it before any stream capture. Every call on a device shares the arrays:
 * calls whose work overlaps on the GPU (other streams, other threads) race
 * and must be serialized by the caller. The addresses are kept for the life
 * of the process: after a cudaDeviceReset (or any other end of the device's
 * primary context) they are stale, and this entry point must not be called
 * again on that device. */
int gb_gpu_attn_decode_noalloc(gb_kernels *k, void *stream, const float *q, const float *kcache,
                               const float *vcache, float *out, int kv_len, int n_heads, int n_kv,
                               int head_dim, float scale);
/* Added (the reference's roadmap "Paged KV cache plus continuous batching",
 * ROADMAP.md:197-202): decode attention for `batch` sequences whose K/V live
 * in pages of a shared pool, k_pool / v_pool = [n_pages][n_kv][page_size]
 * [head_dim] (binary16 when kv_f16, else float32). Sequence b attends over
 * positions [0, seq_lens[b]); position p is row p % page_size of physical
 * page block_table[b * max_pages + p / page_size] (entries outside
 * [0, n_pages) read page 0). q and out are [batch][n_heads][head_dim]
 * float32; per sequence the arithmetic of AttnDecode. head_dim <= 128 and a
 * multiple of 32, at most 8 query heads per KV head. Scratch lives in `k`
 * (grown on demand); calls on `k` must not overlap on the GPU. */
int gb_gpu_attn_decode_paged(gb_kernels *k, void *stream, const float *q, const void *k_pool, const void *v_pool,
                             int kv_f16, const int32_t *block_table, const int32_t *seq_lens, int batch,
                             int max_pages, int n_pages, int page_size, int n_heads, int n_kv, int head_dim,
                             float scale, float *out);
/* (*Kernels).MatVecF16, backend/gpu/gpu.go:126: y[b] = W x[b]. */
int gb_gpu_matvec_f16(gb_kernels *k, void *stream, const uint16_t *w, const float *x, float *y,
                      int rows, int cols, int batch);
/* (*Kernels).MatVecF32, backend/gpu/gpu.go:131. */
int gb_gpu_matvec_f32(gb_kernels *k, void *stream, const float *w, const float *x, float *y,
                      int rows, int cols, int batch);
/* (*Kernels).MatVecQ, backend/gpu/gpu.go:137: W held as raw ggml bytes
 * (Q4_0, Q4_K or Q6_K); cols must be a multiple of the type's block. */
int gb_gpu_matvec_q(gb_kernels *k, void *stream, int typ, const uint8_t *w, const float *x,
                    float *y, int rows, int cols, int batch);
/* gpu.Ones, backend/gpu/gpu.go:157: a new device buffer of n float ones,
 * released with gb_free. */
int gb_gpu_ones(int n, float **out);
/* Releases a buffer returned by gb_gpu_ones. */
int gb_free(void *device_ptr);

/* Added: bit-exact device dequantization of rows [row0, row0+nrows) of a
 * raw ggml [rows][cols] matrix into out[nrows][cols] (the on-device twin of
 * quant.Row, quant/quant.go:135; used for the embedding lookup). */
int gb_gpu_dequant_rows(gb_kernels *k, void *stream, int typ, const uint8_t *w, int rows,
                        int cols, int row0, int nrows, float *out);
/* Added: greedy argmax of n floats on the device into *out (device int32),
 * with model.Argmax's tie rule (model/model.go:376: first maximum wins). */
int gb_gpu_argmax(gb_kernels *k, void *stream, const float *x, int n, int32_t *out);

/* Added (tensor parallelism; the reference is single-GPU, so no reference
 * interface): the partial-sum exchange that follows a row-split GEMV, as a
 * per-op call. bufs and flags are device arrays of `world` device pointers
 * (this rank's own buffers and the peers' buffers mapped into this process,
 * e.g. with CUDA IPC): rank q's partial of `slot` is bufs[q] + slot*dim and
 * its flag is flags[q][slot]. Once every rank's flag equals *step + 1 (step a
 * device word), x[0..n) += the partials summed in rank order and ssq[n/32]
 * receives the per-32 sums of squares of the new x. Each flag wait is bounded
 * by wait_limit polls of ~100 ns (0: the default, about half a second); a
 * wait that runs out skips the sum and ORs GB_DEVERR_TIMEOUT (4) into
 * *status (a device word), leaving the device usable. status NULL: the call
 * waits for the stream and returns GB_ERR_TIMEOUT instead. n is a multiple
 * of 32, n <= dim, world <= 32. */
int gb_gpu_peer_resid(gb_kernels *k, void *stream, int world, const float *const *bufs,
                      const unsigned *const *flags, const unsigned *step, int slot, int dim, float *x, int n,
                      float *ssq, unsigned wait_limit, unsigned *status);
/* Added (tensor parallelism; no reference interface): the exchange the model
 * itself runs after each row-split GEMV. bufs is a HOST array of `world`
 * device pointers (this rank's buffer and the peers' buffers mapped into this
 * process): word bufs[q][slot*dim + c] is rank q's partial of element c as a
 * 64-bit word ((*step + 1) << 32 | the float's bits), written by that rank
 * with no flag. Each element waits (bounded by wait_limit polls of ~100 ns
 * each, 0: the default) until every rank's word carries the tag *step + 1,
 * then x[c] += the values summed in rank order; ssq[n/32] receives the per-32
 * sums of squares of the new x. An element whose wait runs out keeps its x
 * and ORs GB_DEVERR_TIMEOUT (4) into *status (a device word); status NULL:
 * the call waits for the stream and returns GB_ERR_TIMEOUT. n is a multiple
 * of 32, n <= dim, world <= 32. */
int gb_gpu_peer_resid_tagged(gb_kernels *k, void *stream, int world, const unsigned long long *const *bufs,
                             const unsigned *step, int slot, int dim, float *x, int n, float *ssq,
                             unsigned wait_limit, unsigned *status);

/* ---- sampling (added; the reference's roadmap item, ROADMAP.md:42-45) ----
 * One token from a logits vector on the device:
 *  1. the logits of every distinct id among the last repeat_last_n context
 *     tokens are penalised: v <= 0 ? v * repeat_penalty : v / repeat_penalty;
 *  2. temperature <= 0 or top_k == 1: the first maximum (model.Argmax's rule);
 *  3. otherwise s = v / temperature; top_k <= 0 with top_p >= 1 samples the
 *     whole vocabulary in index order; else the candidates are the
 *     min(top_k > 0 ? top_k : 1024, 1024) largest, sorted (value
 *     descending, index ascending), cut to the shortest prefix whose
 *     probability reaches top_p;
 *  4. the draw u in [0,1) is splitmix64 of (seed, counter), 24 bits.
 * The exact float32 operations (and the association of every sum) are
 * fixed, so a host restatement picks the same token bit for bit. */
typedef struct {
  float temperature;     /* <= 0: greedy */
  int top_k;             /* <= 0: no limit */
  float top_p;           /* >= 1: no nucleus cut */
  float repeat_penalty;  /* 1: none */
  int repeat_last_n;     /* context tokens the penalty looks back over (<= 0: none) */
  int reserved;          /* 0 */
  uint64_t seed;
} gb_sample_params;

/* Largest vocabulary the sampler accepts. */
#define GB_SAMPLE_MAX_VOCAB (1 << 20)

/* Sample one token from logits[n] (device) into *out (device int32).
 * recent[n_recent] (device, may be NULL when n_recent == 0) holds the context
 * ids, oldest first; the penalty looks at the last repeat_last_n of them.
 * counter selects the draw (use the position). */
int gb_gpu_sample(gb_kernels *k, void *stream, const float *logits, int n, const gb_sample_params *p,
                  const int32_t *recent, int n_recent, uint64_t counter, int32_t *out);

/* ---- model.Linear with the B200 tiled layout ----------------------------- */
typedef struct gb_linear gb_linear;
/* uploadLinear, model/model.go:77: uploads a [rows][cols] matrix given as
 * raw ggml bytes on the host and repacks it on the device into 32-row
 * tiles. Supported: Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32 with cols a multiple of 256. */
int gb_linear_upload(int device, int typ, const void *host_bytes, size_t nbytes, int rows,
                     int cols, gb_linear **out);
/* (*Linear).MatVec, model/model.go:109 for batch 1: y[rows] = W x[cols]
 * (x and y device pointers). Launched with programmatic dependent launch:
 * the weights start streaming while the stream's previous kernel finishes;
 * x is read and y written only after it has completed. Calls on one
 * gb_linear must not overlap on the GPU (they share its scratch). */
int gb_linear_matvec(gb_linear *l, void *stream, const float *x, float *y);
/* Added: the prefill GEMM on the tensor cores (tcgen05), the batched
 * MatVecQ of the reference's roadmap (ROADMAP.md:99-101): y[T][rows] =
 * x[T][cols] W^T with x binary16 on the device (row stride cols, 16-byte
 * aligned) and y float32 (row stride rows). W's elements are the
 * reference's float32 element values rounded to binary16; products
 * accumulate in float32. When the weight tiles alone are too few to fill the
 * GPU, K is split and fp32 partials are summed in a fixed order by a second
 * kernel (deterministic); their scratch is allocated by the first call that
 * needs it (after a device synchronisation). */
int gb_linear_matmul_f16(gb_linear *l, void *stream, const uint16_t *x, int T, float *y);
/* Added: the binary16 copy of the Linear's weights (the values the matmul
 * decodes them to; 2 bytes per weight) for gb_linear_matmul_f16 to read by
 * TMA instead of decoding the quantized tiles each call; bit-identical
 * results. *bytes (may be NULL) receives its size. */
int gb_linear_cache_f16_weights(gb_linear *l, size_t *bytes);
/* Bytes of the tiled weight buffer and the type's algorithmic bytes. */
int gb_linear_info(const gb_linear *l, int *typ, int *rows, int *cols, size_t *weight_bytes);
int gb_linear_free(gb_linear *l);

/* ---- model ------------------------------------------------------------- */
typedef struct gb_model gb_model;

typedef struct {
  int layers, dim, ffn, heads, kv_heads, head_dim, vocab, ctx_len; /* model.Config, model/model.go:20 */
  float rope_base, eps;
  int max_len;   /* KV positions allocated (Model.MaxLen, model/model.go:137) */
  int kv_f16;    /* 1 = binary16 KV cache, 0 = float32 */
  int tp_rank, tp_world;
} gb_config;

typedef struct {
  int device;        /* CUDA device ordinal */
  int max_len;       /* <= 0 or above the file's context_length: context_length (model.go:165) */
  int kv_f16;        /* 1 = fp16 KV cache (B200 default), 0 = the reference's float32 cache */
  int use_graph;     /* 1 = one CUDA graph per token (default), 0 = eager launches */
  int tp_rank;       /* tensor-parallel rank (0 for one GPU) */
  int tp_world;      /* tensor-parallel world size (1 for one GPU) */
  const uint8_t *nccl_id; /* 128-byte ncclUniqueId shared by all ranks when tp_world > 1 */
} gb_model_opts;

/* Defaults: device 0, max_len 0, kv_f16 1, use_graph 1, rank 0, world 1. */
void gb_model_opts_default(gb_model_opts *o);

/* model.Load, model/model.go:160, from a GGUF file on disk (mmap'd). */
int gb_model_load(const char *gguf_path, const gb_model_opts *opts, gb_model **out);
/* model.Load from a GGUF image in host memory (gguf.Parse, gguf/gguf.go:62);
 * the image is only read during the call. */
int gb_model_load_mem(const void *gguf, size_t len, const gb_model_opts *opts, gb_model **out);
/* The Config fields of the loaded model (model/model.go:20-32). */
int gb_model_config(const gb_model *m, gb_config *c);
/* (*Model).Forward, model/model.go:313: logits of `token` at `pos` copied
 * into host_logits[vocab] (on rank 0 when tp_world > 1; other ranks may
 * pass NULL). Same validation and errors as the reference. A page-locked
 * host_logits (cudaHostAlloc / registered) receives the device copy
 * directly; pageable memory goes through an internal pinned buffer. */
int gb_model_forward(gb_model *m, int32_t token, int pos, float *host_logits);
/* Added: one greedy step entirely on the device; only the next token id
 * comes back to the host (model.Argmax applied on the device). */
int gb_model_next(gb_model *m, int32_t token, int pos, int32_t *next);
/* Added: n greedy steps from (token, pos) with no host round trip between
 * them; out_tokens[n] receives the generated ids. */
int gb_model_generate(gb_model *m, int32_t token, int pos, int n, int32_t *out_tokens);
/* Added, the three parts of gb_model_generate for callers that time or
 * overlap the device work: stage (token, pos) on the device (stream-ordered,
 * no host wait); run n greedy steps from the device-resident token and
 * position (graph replays, no host wait); wait and copy the ids generated at
 * positions [pos0, pos0+n) (checks the device status word). */
int gb_model_start(gb_model *m, int32_t token, int pos);
int gb_model_decode_async(gb_model *m, int n);
int gb_model_read_tokens(gb_model *m, int pos0, int n, int32_t *out_tokens);
/* Added (the reference's roadmap "Batched prefill", ROADMAP.md:36-41): feed
 * tokens[0..n) at positions pos0..pos0+n-1. The first n-1 go through every
 * layer at once (tensor-core GEMMs over binary16 activations and weights with
 * float32 accumulation, causal attention over the cache; chunks of up to 512
 * tokens), writing their K/V; the last goes through the decode step, whose
 * logits are copied to host_logits[vocab] (NULL: not copied; under tensor
 * parallelism every rank makes the call with the same tokens, the o and down
 * partials are summed by NCCL all-reduces, and rank 0 receives the logits). */
int gb_model_prefill(gb_model *m, const int32_t *tokens, int n, int pos0, float *host_logits);
/* Added: keep a binary16 copy of every weight matrix on the device (the
 * values the tensor-core GEMMs decode the quantized weights to, so results
 * are bit-identical) and have gb_model_prefill and gb_engine_step read it by
 * TMA instead of decoding the quantized tiles each call. Costs 2 bytes per
 * weight of device memory (about 16 GB for an 8B model); *bytes (may be NULL)
 * receives the amount this call allocated (0 once the copy exists). Fails with GB_ERR_UNSUPPORTED, leaving the model as it
 * was, when free device memory is short of it plus 1 GiB. The decode step
 * (gb_model_forward / next / generate) keeps the quantized weights. */
int gb_model_cache_f16_weights(gb_model *m, size_t *bytes);
/* ---- continuous batching (added; the reference's roadmap "Paged KV cache
 * plus continuous batching", ROADMAP.md:197-202) ---------------------------
 * An engine over a loaded model (one GPU) decodes many sequences at once.
 * Each sequence owns pages of a paged KV pool (per layer
 * [n_pages][n_kv][page_size][head_dim] binary16) taken from a free list as it
 * grows and returned by gb_engine_release. A step feeds one token to each of
 * n listed sequences (at their next positions) and runs them as the rows of
 * one batched pass: the prefill's tensor-core GEMMs (binary16 operands, f32
 * accumulate), RoPE and K/V append through the page tables, the paged
 * attention, then the output RMSNorm and lm_head; logits agree with the
 * one-sequence decode to the prefill's tolerance. Sequences may join and
 * leave between steps. The engine shares the model's stream and prefill
 * workspace: do not interleave its calls with the model's on other threads. */
typedef struct gb_engine gb_engine;
/* page_size positions per page, n_pages pages per layer, at most max_batch
 * (<= 512) sequences per step. */
int gb_engine_create(gb_model *m, int page_size, int n_pages, int max_batch, gb_engine **out);
/* A new, empty sequence; its id is reused after gb_engine_release. */
int gb_engine_add(gb_engine *e, int *seq_id);
int gb_engine_release(gb_engine *e, int seq_id);
/* Positions fed so far (-1: no such sequence); free pages of the pool. */
int gb_engine_seq_len(const gb_engine *e, int seq_id);
int gb_engine_free_pages(const gb_engine *e);
/* Rows (seq_ids[t], tokens[t]) for t in [0, n), n <= max_batch, each a live
 * sequence. A sequence listed k times feeds k tokens at its next k positions
 * in the order listed (a prompt chunk in one step); each row attends to its
 * sequence's positions up to its own. The logits of each row are copied to
 * host_logits[n][vocab] and the first maximum of each row (model.Argmax's
 * rule) to next[n]; either may be NULL. Fails (GB_ERR_UNSUPPORTED) without
 * changing any sequence when the pool has too few free pages for the step,
 * and (GB_ERR_INVALID) when a sequence would pass the cache's length. */
int gb_engine_step(gb_engine *e, int n, const int32_t *seq_ids, const int32_t *tokens, float *host_logits,
                   int32_t *next);
int gb_engine_free(gb_engine *e);

/* Added: the token rule of gb_model_next / generate / decode_async. NULL
 * (the default) is greedy model.Argmax; otherwise the sampler above with
 * counter = the position of the step and the penalty window = the tokens fed
 * at the last repeat_last_n positions (prompt included). One GPU only
 * (GB_ERR_UNSUPPORTED under tensor parallelism). */
int gb_model_set_sampler(gb_model *m, const gb_sample_params *p);
/* Added: fill KV positions [0, n_pos) of every layer with the seeded N(0,1)
 * values of gb_synth_kv_normal (rounded to the cache type). */
int gb_model_fill_kv_normal(gb_model *m, uint64_t seed, int n_pos);
/* Added: copy cache rows [pos0, pos0+n) of one layer to the host in the
 * reference's layout ([n][kv_heads*head_dim] float32), for parity tests. */
int gb_model_read_kv(gb_model *m, int layer, int pos0, int n, float *k_out, float *v_out);
/* Added: the stream the model launches on (cudaStream_t). */
void *gb_model_stream(gb_model *m);
/* Added: per-kernel-class device time of one eager decode step at pos
 * (token from the host), in ms, summed over the step's launches:
 * out[0] qkv, [1] attention, [2] o-proj, [3] gate/up, [4] down, [5] lm_head,
 * [6] everything else; launches[7] receives the launch counts. */
int gb_model_profile_step(gb_model *m, int32_t token, int pos, float *ms_out, int *launches);
/* Added: algorithmic HBM bytes of one decode step at kv length kv_len, and
 * the weight bytes of the dominant GEMV launch (gate/up) of one layer. */
int gb_model_step_bytes(const gb_model *m, int kv_len, double *bytes_per_token,
                        double *gateup_bytes_per_launch);
/* Number of kernel launches one decode step makes. */
int gb_model_launches_per_step(const gb_model *m);
/* (*Model).Close, model/model.go:387. */
int gb_model_close(gb_model *m);

/* model.Argmax, model/model.go:376 (host; first maximum wins). */
int32_t gb_argmax(const float *logits, int64_t n);

/* ---- GGUF container (the gguf package the loader reads through) ---------- */
typedef struct gb_gguf gb_gguf;
/* gguf.Parse, gguf/gguf.go:62: parse an image held in memory (the image is
 * not copied and must outlive the handle). */
int gb_gguf_parse(const void *data, size_t len, gb_gguf **out);
/* gguf.Open, gguf/open_unix.go:13: mmap and parse a file. */
int gb_gguf_open(const char *path, gb_gguf **out);
/* (*File).Close, gguf/gguf.go:135. */
int gb_gguf_close(gb_gguf *f);
/* File.Version / File.Alignment, gguf/gguf.go:24-26; number of keys and tensors. */
int gb_gguf_header(const gb_gguf *f, uint32_t *version, uint32_t *alignment, int *n_kv,
                   int *n_tensors);
/* (*File).Uint / Float / String with a default, gguf/gguf.go:154-176. */
uint64_t gb_gguf_uint(const gb_gguf *f, const char *key, uint64_t def);
double gb_gguf_float(const gb_gguf *f, const char *key, double def);
/* Copies the string value (NUL-terminated, truncated to cap) or def. */
int gb_gguf_string(const gb_gguf *f, const char *key, const char *def, char *out, int cap);
/* Name of key i (file order) and its value type; NULL when i is out of range. */
const char *gb_gguf_key(const gb_gguf *f, int i, int *value_type);
/* Array value: element type and length (0 if key is not an array); element
 * j as float64 / as string. Value.Floats / Value.Strings, gguf/gguf.go:273-298. */
int gb_gguf_array_len(const gb_gguf *f, const char *key, int *elem_type);
double gb_gguf_array_float(const gb_gguf *f, const char *key, int j);
int gb_gguf_array_string(const gb_gguf *f, const char *key, int j, char *out, int cap);
/* (*File).Tensor, gguf/gguf.go:145 + TensorInfo fields: returns GB_OK and
 * fills type, ndims, dims (ggml order, innermost first), offset within the
 * data section, byte size and a pointer to the bytes; GB_ERR_INVALID when
 * the tensor does not exist. Tensor i by file order with gb_gguf_tensor_at. */
int gb_gguf_tensor(const gb_gguf *f, const char *name, int *type, int *ndims, uint64_t dims[4],
                   uint64_t *offset, uint64_t *nbytes, const void **data);
const char *gb_gguf_tensor_at(const gb_gguf *f, int i);

/* ---- tensor parallelism ------------------------------------------------- */
/* A fresh ncclUniqueId (128 bytes) for rank 0 to share with the others. */
int gb_tp_unique_id(uint8_t out[128]);

/* ---- synthetic GGUF models (seeded, counter-based) ----------------------- */
typedef struct {
  int layers, dim, ffn, heads, kv_heads, head_dim, vocab, ctx_len;
  float rope_base, eps;
  int mix;        /* 0 = all Q4_0 with tied head; 1 = Q4_K_M mix (Q6_K attn_v,
                     even-layer ffn_down and output); 2 = all Q4_K; 3 = all Q6_K;
                     4 = all Q8_0; 5 = all F16; 6 = Q5_K_M mix (as 1 with Q5_K
                     in place of Q4_K) */
  uint64_t seed;
} gb_synth_spec;
/* Fills spec with a BASELINE preset: 1 = Llama-3.2-1B Q4_0, 3 = 3B Q4_K_M,
 * 8 = 8B Q4_K_M, 70 = 70B Q4_K_M. */
int gb_synth_preset(int preset, gb_synth_spec *spec);
/* Builds the GGUF image of a synthetic model in host memory (gb_synth_free). */
int gb_synth_model(const gb_synth_spec *spec, void **gguf, size_t *len);
/* Writes the same image to a file. */
int gb_synth_model_file(const gb_synth_spec *spec, const char *path);
void gb_synth_free(void *gguf);
/* Raw bytes of one synthetic [rows][cols] matrix of typ (the GEMV sweep),
 * generated like the model tensors; buf must hold rows*RowBytes(cols). */
int gb_synth_matrix(int typ, int rows, int cols, uint64_t seed, uint32_t tensor_id,
                    float scale_sigma, void *buf);
/* Seeded N(0,1) float32 vector (activations). */
int gb_synth_normal(uint64_t seed, uint32_t stream_id, int64_t n, float *out);
/* The N(0,1) KV prefill of one layer: k and v [n][kv_dim] for positions
 * [pos0, pos0+n), rounded through binary16 when f16 != 0. */
int gb_synth_kv_normal(uint64_t seed, int layer, int pos0, int n, int kv_dim, int f16,
                       float *k, float *v);

#ifdef __cplusplus
}
#endif
#endif
