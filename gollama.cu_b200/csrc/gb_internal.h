// gb_internal.h -- host-side internals shared by the library's translation
// units: error reporting, kernel launch entry points, GGUF reader/writer.
#pragma once

#include <cuda.h>  // CUtensorMap (the encoder is reached through cudaGetDriverEntryPoint)
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <string>
#include <vector>

#include "../../include/gollama_b200.h"
#include "gb_formats.h"

// ---- errors: each entry point returns a status and leaves a message in
// the calling thread's slot, worded like the reference's wrapped Go errors.
int gb_fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int gb_cuda_fail(cudaError_t e, const char *what);
void gb_clear_error();

#define GB_CUDA(call, what)                              \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return gb_cuda_fail(e_, what); \
  } while (0)

// ---- tiled GEMV (gb_gemv.cu)
enum GbEpi {
  GB_EPI_PLAIN = 0,   // y[r] = W x
  GB_EPI_QKV = 1,     // RoPE q,k; q -> qbuf, k,v -> KV cache at *pos
  GB_EPI_RESID = 2,   // x[r] += y; per-32 sums of squares for the next RMSNorm
  GB_EPI_SWIGLU = 3,  // gate/up pairs -> act = silu(g)*u
  GB_EPI_LOGITS = 4,  // logits[r] = y; argmax candidates; last CTA -> token
  GB_EPI_PARTIAL = 5, // tensor parallel: this rank's partial y, tagged with the step, into its peer slot
};

// Tensor-parallel exchange over peer memory; every buffer is mapped into the
// other ranks' address spaces (CUDA IPC). The row-split GEMVs' partials go to
// `my_tbuf` as 64-bit words tagged with epoch + 1, which the peers read with no
// flag (peer_resid_tagged_kernel). The lm_head's argmax key goes to `my_buf`
// and is published by flag[s] = epoch + 1 (system-scope release); the per-op
// flag exchange (gb_gpu_peer_resid) uses the same pair. `epoch` counts decode
// steps, only grows, and is the same on every rank.
struct GbPeer {
  int world = 1, rank = 0, dim = 0;
  const float *const *bufs = nullptr;     // device array [world]: every rank's partials
  const unsigned *const *flags = nullptr; // device array [world]: every rank's flags
  float *my_buf = nullptr;                // this rank's partials [slots][dim]
  unsigned *my_flag = nullptr;            // this rank's flags [slots]
  const unsigned *epoch = nullptr;        // device step counter
  // this rank's partials of the row-split GEMVs as tagged words [slots][dim]:
  // (step + 1) << 32 | float bits, read by the peers with no flag
  unsigned long long *my_tbuf = nullptr;
  unsigned wait_limit = 1u << 22;         // polls of a peer flag (~100 ns each) before a wait gives up
};

struct GbGemvPlan {
  int warps = 8;    // warps per CTA
  int rb = 1;       // row tiles per CTA
  int ks = 1;       // K splits across CTAs
  int stages = 3;   // sb-blocks in flight per warp
};

struct GbEpiArgs {
  // QKV
  float *q_out = nullptr;
  void *kcache = nullptr, *vcache = nullptr;  // head-major caches
  int q_rows = 0, kv_rows = 0, head_dim = 0, max_len = 0, kv_f16 = 1;
  const double *rope_cs = nullptr;  // [max_len][head_dim/2][2] (cos, sin)
  const int32_t *pos = nullptr;
  // RESID: x += y and per-row-block sums of squares of the new x
  float *x = nullptr;
  float *ssq = nullptr;
  // LOGITS / PLAIN / SWIGLU output
  float *y = nullptr;
  unsigned long long *best = nullptr;     // running argmax key (zero between launches)
  unsigned *counter = nullptr;            // finished row-blocks (zero between launches)
  int32_t *token_out = nullptr;   // argmax result (device)
  int32_t *token_hist = nullptr;  // optional history slot base ([max_len]); indexed by *pos
  int row_offset = 0;             // global index of local row 0 (vocab shard)
  int vocab_total = 0;
  unsigned *err = nullptr;
  // K-split scratch
  float *part = nullptr;          // [ntiles][ks][32]
  unsigned *tile_counter = nullptr;
  // PARTIAL (and LOGITS under tensor parallelism): peer exchange slot
  GbPeer peer;
  int peer_slot = -1;
};

struct GbGemvArgs {
  const uint8_t *w = nullptr;  // tiled weights
  int type_a = GB_T_Q4_K, type_b = GB_T_Q4_K;
  int split_tile = 1 << 30;    // tiles >= split_tile use type_b
  int rows = 0, ntiles = 0, nsb = 0;
  const float *in_x = nullptr;    // input vector [nsb*256] (float, from the preceding kernel)
  const float *in_w = nullptr;    // RMSNorm weights when the input is normalised in the prologue
  const float *in_ssq = nullptr;  // per-32 sums of squares of in_x (with in_w)
  float eps = 1e-5f;
  int epi = GB_EPI_PLAIN;
  GbEpiArgs e;
};

int gb_gemv_launch(const GbGemvArgs &a, const GbGemvPlan &p, cudaStream_t st, bool pdl);
GbGemvPlan gb_gemv_plan(int ntiles, int nsb, int epi, int sms);
size_t gb_tiled_bytes(int typ, int rows, int cols);
int gb_repack_launch(int typ, const uint8_t *raw, int rows, int cols, uint8_t *tiled,
                     cudaStream_t st);
// Floats of the GEMV scratch (GbEpiArgs::part) a caller allocates: split-row
// partials and the fourth limb planes of outlier input blocks.
int gb_gemv_scratch_floats(int ntiles, const GbGemvPlan &p);

// ---- attention (gb_attn.cu)
struct GbAttnArgs {
  const float *q = nullptr;
  const void *k = nullptr, *v = nullptr;
  int kv_f16 = 0;
  // element strides (in elements of the cache type)
  long long k_sh = 0, k_sd = 0, k_st = 0;  // head, 16-byte dim chunk, position
  long long v_sh = 0, v_st = 0;            // head, position (dims contiguous)
  long long v_sd = 0;                      // 16-byte dim chunk (fp16 model cache only)
  int n_heads = 0, n_kv = 0, head_dim = 0;
  float scale = 1.f;
  int kv_len = 0;                // used when kv_len_pos is null
  const int32_t *kv_len_pos = nullptr;  // kv_len = *kv_len_pos + 1
  int max_len = 0;
  int splits = 1;
  float *out = nullptr;          // [n_heads*head_dim]
  float *part = nullptr;         // [n_kv][splits][group][head_dim+4]
  unsigned *counter = nullptr;   // [n_kv], zero between launches
  unsigned *err = nullptr;
  // fp16 model caches: 4-D tensor maps of K and V ([head][dim chunk][position][8 halves]),
  // box of one head x all chunks x 128 positions, for whole 128-position sub-chunks
  int tmap = 0;
  CUtensorMap tk, tv;
};
int gb_attn_launch(const GbAttnArgs &a, cudaStream_t st, bool pdl);
// Encode the tensor maps of one layer's fp16 K and V caches (the model layout).
int gb_attn_tensor_maps(const void *k, const void *v, int n_kv, int head_dim, int max_len, CUtensorMap *tk,
                        CUtensorMap *tv);
int gb_attn_splits(int n_kv, int max_len, int sms);
size_t gb_attn_part_floats(int n_kv, int splits, int group, int head_dim);

// ---- misc kernels (gb_ops.cu)
// Embedding row of *token into x, with per-32 sums of squares (first RMSNorm).
int gb_embed_launch(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *token,
                    int vocab, float *x, float *ssq, unsigned *err, int32_t *fed, const int32_t *pos, int max_len,
                    cudaStream_t st, bool pdl);
// x += y with per-32 sums of squares: the residual after a collective.
int gb_resid_launch(float *x, const float *y, int n, float *ssq, cudaStream_t st, bool pdl);
int gb_add_launch(const float *a, const float *b, float *out, int n, cudaStream_t st);
// Tensor parallel: wait for every rank's partial in peer slot `slot`, then
// x += sum of the partials (rank order, identical on every rank) with per-32
// sums of squares.
// Every rank's tagged partial buffer (this rank's own and the peers' mapped
// ones), passed by value so the exchange kernel reads the pointers from its
// parameters.
constexpr int kGbMaxWorld = 32;
struct GbTagTable {
  const unsigned long long *w[kGbMaxWorld];
};
int gb_peer_resid_tagged_launch(const GbTagTable &t, int world, const unsigned *step, unsigned wait_limit, int slot,
                                int dim, float *x, int n, float *ssq, unsigned *err, cudaStream_t st, bool pdl);
int gb_peer_resid_launch(const GbPeer &p, int slot, float *x, int n, float *ssq, unsigned *err,
                         cudaStream_t st, bool pdl);
// Tensor parallel: wait for every rank's argmax key in peer slot `slot` and
// reduce them to the token.
int gb_peer_argmax_launch(const GbPeer &p, int slot, int32_t *token, int32_t *hist, const int32_t *pos,
                          int max_len, unsigned *err, cudaStream_t st, bool pdl);
// Advance the position (and the tensor-parallel step counter when non-null).
int gb_advance_pos_launch(int32_t *pos, unsigned *epoch, cudaStream_t st);

// gb_prefill.cu: the batched prefill kernels. The GEMM multiplies T token
// rows of a binary16 activation (TMA map tmap_a over [T][nsb*256]) by a
// tiled weight matrix on the tensor cores: PLAIN y[T][ldy] = A W^T, RESID
// y += A W^T, SWIGLU act[T][ld_act] = silu(A Wg^T) * (A Wu^T) over gate/up
// pairs (rows and ntiles then count one half).
struct GbTcGemm {
  const uint8_t *w = nullptr;
  int type_a = 0, type_b = 0, split_tile = 1 << 30;
  int rows = 0, ntiles = 0, nsb = 0;
  int epi = GB_EPI_PLAIN;
  int T = 0;
  float *y = nullptr;
  int ldy = 0;
  __half *act = nullptr;
  int ld_act = 0;
  unsigned *err = nullptr;
  float *part = nullptr;       // split-K partials (may be null: no split)
  size_t part_floats = 0;
  CUtensorMap tmap_a;
  const __half *w16 = nullptr;  // the matrix's binary16 copy (gb_tc_f16_weights_launch) or null
  CUtensorMap tmap_b;           // its tensor map, with w16
  bool a16 = false;             // tmap_a16 is set: the activation with 16-row boxes
  CUtensorMap tmap_a16;
};
struct GbTcPlan {
  int mt = 1, splits = 1;
  size_t part_floats = 0;
  bool swap = false;  // tokens as the MMA's N (few token rows, binary16 weight copy)
};
GbTcPlan gb_tc_gemm_plan(const GbTcGemm &a, int sms);
int gb_tmap_f16_rows(const void *base, int rows, int cols, CUtensorMap *map, int box_rows = 128);
int gb_tc_gemm_launch(const GbTcGemm &a, cudaStream_t st);
// The binary16 copy of a GEMM's weights, the values the GEMM decodes to:
// gb_tc_f16_rows(a) rows of a.nsb * 256 columns; writes its tensor map.
size_t gb_tc_f16_rows(const GbTcGemm &a);
int gb_tc_f16_weights_launch(const GbTcGemm &a, __half *w16, CUtensorMap *map, cudaStream_t st);
int gb_embed_rows_launch(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *tokens, int T, int vocab,
                         float *x, int32_t *fed, int pos0, int max_len, unsigned *err, cudaStream_t st);
int gb_rmsnorm_rows_f16_launch(const float *x, const float *w, int rows, int n, float eps, __half *out,
                               cudaStream_t st);
int gb_rope_kv_launch(const float *qkv, int T, int q_rows, int kv_rows, int hd, const double *rope_cs, int pos0,
                      int max_len, int kv_f16, float *q_out, void *kcache, void *vcache, cudaStream_t st);
int gb_attn_prefill_launch(const float *q, int T, int pos0, int n_heads, int n_kv, int hd, const void *kcache,
                           const void *vcache, int kv_f16, int max_len, __half *out, cudaStream_t st);

// gb_paged.cu: batched decode attention through per-sequence page tables.
size_t gb_paged_part_floats(int B, int n_kv, int S, int G, int hd);
int gb_attn_paged_launch(const float *q, const void *k_pool, const void *v_pool, int kv_f16, const int32_t *block_table,
                         const int32_t *seq_lens, int B, int max_pages, int n_pages, int page_size, int n_heads,
                         int n_kv, int hd, float scale, float *out, __half *out16, float *part, unsigned *counter,
                         int S, unsigned *err, cudaStream_t st, const int32_t *groups = nullptr, int n_groups = 0);
// Rows of one sequence a paged-attention row group may hold (query heads per KV head G).
int gb_attn_paged_group_rows(int G);

int gb_rope_kv_paged_launch(const float *qkv, int T, int q_rows, int kv_rows, int hd, const double *rope_cs,
                            const int32_t *pos, const int32_t *table, int max_pages, int page_size, int n_pages,
                            int max_len, float *q_out, uint16_t *kpool, uint16_t *vpool, unsigned *err,
                            cudaStream_t st);
int gb_f32_to_f16_launch(const float *x, __half *y, size_t n, cudaStream_t st);
int gb_argmax_rows_launch(const float *x, int rows, int n, int32_t *out, cudaStream_t st);

// gb_sample.cu: one token from logits[n]; parameters by value (p_host) or
// from device memory (p_dev, for graph replays); the penalty window is
// recent[n_recent] or, for the model, fed[pos-N+1..pos]; counter = *pos when
// pos is given. Writes *out and, with gen, gen[*pos].
typedef gb_sample_params GbSampleParams;
constexpr int kSampleMaxVocab = GB_SAMPLE_MAX_VOCAB;
int gb_sample_launch(const float *logits, int n, const GbSampleParams *p_host, const GbSampleParams *p_dev,
                     const int32_t *recent, int n_recent, const int32_t *fed, const int32_t *pos, int max_len,
                     unsigned long long counter, int32_t *out, int32_t *gen, unsigned *err, cudaStream_t st);

// ---- GGUF (gb_gguf.cpp): reader restating gguf/gguf.go:62 Parse and
// writer restating gguf/writer.go.
struct GbTensor {
  std::string name;
  std::vector<uint64_t> dims;  // ggml order, innermost first
  int type = 0;
  uint64_t offset = 0;
  const uint8_t *data = nullptr;
  uint64_t bytes = 0;
  int rows() const { return dims.size() >= 2 ? (int)dims[1] : 1; }
  int cols() const { return dims.empty() ? 0 : (int)dims[0]; }
  uint64_t numel() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct GbValue {
  int type = 0;  // gguf value type
  uint64_t u = 0;
  double f = 0;
  std::string s;
  int elem = 0;
  std::vector<GbValue> arr;
  // gguf/gguf.go:223 IsInt: the eight integer value types.
  bool is_int() const { return (type >= 0 && type <= 5) || type == 10 || type == 11; }
};

struct GbGguf {
  uint32_t version = 0, alignment = 32;
  std::vector<std::pair<std::string, GbValue>> kv;
  std::vector<GbTensor> tensors;
  const uint8_t *data = nullptr;
  size_t len = 0;
  uint64_t data_offset = 0;
  // mmap bookkeeping (Open)
  void *map = nullptr;
  size_t map_len = 0;
  ~GbGguf();
  const GbValue *get(const std::string &k) const;
  uint64_t get_uint(const std::string &k, uint64_t def) const;
  double get_float(const std::string &k, double def) const;
  std::string get_string(const std::string &k, const std::string &def) const;
  const GbTensor *tensor(const std::string &name) const;
};
// Parse a GGUF image (not copied). Returns nullptr and sets the error.
GbGguf *gb_gguf_parse(const uint8_t *data, size_t len);
GbGguf *gb_gguf_open(const char *path);

struct GbGgufWriter {
  std::vector<std::pair<std::string, GbValue>> kv;
  struct T {
    std::string name;
    std::vector<uint64_t> dims;
    int type = 0;
    uint64_t bytes = 0;
    std::vector<uint8_t> data;  // may stay empty until the image is filled
  };
  std::vector<T> tensors;
  uint32_t alignment = 32;
  void set_u32(const std::string &k, uint32_t v);
  void set_f32(const std::string &k, float v);
  void set_str(const std::string &k, const std::string &v);
  int add_tensor(const std::string &name, const std::vector<int> &shape, int type,
                 std::vector<uint8_t> &&data);
  // Header bytes (padded to the alignment), per-tensor data offsets and the
  // total image size; tensor bytes go at header.size() + offsets[i].
  std::vector<uint8_t> layout(std::vector<uint64_t> *offsets, uint64_t *total) const;
  std::vector<uint8_t> write() const;
};

// ---- synthetic data (gb_synth.cpp)
uint64_t gb_splitmix64(uint64_t *state);
uint64_t gb_stream_seed(uint64_t seed, uint64_t tensor, uint64_t block);
int gb_host_threads();
