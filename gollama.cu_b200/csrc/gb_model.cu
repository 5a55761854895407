// gb_model.cu -- the decode-step runtime: model.Load / (*Model).Forward /
// Close (model/model.go:160-392) on B200, plus model.Linear (model/model.go:67-126).
//
// Load reads the GGUF (mmap'd file or a memory image), checks the config
// like model.ConfigFrom (model/model.go:35), uploads each quantized matrix
// and repacks it on the device into the 32-row tiled layout (gb_formats.h),
// uploads float32 norms, and allocates head-major KV caches. Tensor
// parallelism (tp_world > 1): q/k/v and gate/up rows are split by heads /
// FFN rows, o and down by input columns, the lm_head by vocabulary rows;
// the two row-split projections of each layer are summed with an NCCL
// all-reduce and the greedy token is the maximum of the per-rank argmax
// keys (one 8-byte all-gather).
//
// One decode step is 5 launches per layer plus 3 (embedding, lm_head with
// the argmax, position advance), each a persistent kernel launched with
// programmatic dependent launch so the next kernel's weight copies start
// while the previous one finishes; the whole step is captured once into a
// CUDA graph whose kernels read the token and position from device memory.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "gb_internal.h"

// ---- NCCL through dlopen: the library loads without NCCL on one GPU, and
// reuses the libnccl.so.2 a host process (e.g. torch) already mapped.
namespace {
struct NcclApi {
  void *h = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  const char *(*getErrorString)(ncclResult_t) = nullptr;
};
NcclApi *nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    api.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (api.h) {
      api.getUniqueId = (decltype(api.getUniqueId))dlsym(api.h, "ncclGetUniqueId");
      api.commInitRank = (decltype(api.commInitRank))dlsym(api.h, "ncclCommInitRank");
      api.allReduce = (decltype(api.allReduce))dlsym(api.h, "ncclAllReduce");
      api.allGather = (decltype(api.allGather))dlsym(api.h, "ncclAllGather");
      api.commDestroy = (decltype(api.commDestroy))dlsym(api.h, "ncclCommDestroy");
      api.getErrorString = (decltype(api.getErrorString))dlsym(api.h, "ncclGetErrorString");
    }
  }
  return api.h && api.commInitRank && api.allReduce && api.allGather ? &api : nullptr;
}
#define GB_NCCL(call, what)                                                                  \
  do {                                                                                       \
    ncclResult_t r_ = (call);                                                                \
    if (r_ != ncclSuccess)                                                                   \
      return gb_fail(GB_ERR_NCCL, "%s: %s", what,                                            \
                     nccl()->getErrorString ? nccl()->getErrorString(r_) : "nccl error");    \
  } while (0)

float host_half(uint16_t h) {
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

uint16_t host_f16(float x) {
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

const char *tname(int t) {
  switch (t) {
    case GB_T_F32: return "F32";
    case GB_T_F16: return "F16";
    case GB_T_Q4_0: return "Q4_0";
    case GB_T_Q8_0: return "Q8_0";
    case GB_T_Q4_K: return "Q4_K";
    case GB_T_Q5_K: return "Q5_K";
    case GB_T_Q6_K: return "Q6_K";
    case GB_T_BF16: return "BF16";
  }
  return "?";
}

// A tiled matrix on the device (possibly several row segments concatenated).
struct Tiled {
  uint8_t *w = nullptr;
  int type_a = 0, type_b = 0, split_tile = 1 << 30;
  int rows = 0, cols = 0, ntiles = 0, nsb = 0;
  size_t bytes = 0;
  bool owned = true;
  __half *w16 = nullptr;  // binary16 copy for the tensor-core GEMMs (gb_model_cache_f16_weights)
  CUtensorMap map16;
};

enum { K_QKV = 0, K_ATTN, K_O, K_GU, K_DOWN, K_HEAD, K_OTHER, K_CLASSES };

// Tensor maps of one binary16 activation buffer: 128-row boxes (the
// dequantizing GEMM's token tiles) and 16-row boxes (the few-token GEMM).
struct AMap {
  CUtensorMap a128, a16;
};

}  // namespace

struct gb_linear {
  int device = 0;
  Tiled t;
  float *part = nullptr;
  unsigned *tile_counter = nullptr;
  float *mm_part = nullptr;  // split-K partials of matmul_f16 (grown on demand)
  size_t mm_part_floats = 0;
};

struct gb_model {
  gb_config c{};
  gb_model_opts o{};
  int q_local = 0, kv_local = 0, ffn_local = 0, vocab_local = 0, vocab_off = 0;
  int embd_type = 0, embd_nsb = 0;
  struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    Tiled qkv, wo, gu, down;
    void *kc = nullptr, *vc = nullptr;
    bool tmap = false;  // fp16 caches: tensor maps of K and V for the attention's TMA
    CUtensorMap tk, tv;
  };
  std::vector<Layer> layers;
  Tiled embd, head;
  float *out_norm = nullptr;
  double *rope_cs = nullptr;
  // work
  float *x = nullptr, *q = nullptr, *attn = nullptr, *logits = nullptr, *logits_full = nullptr;
  float *act = nullptr;  // SwiGLU output [ffn_local]
  float *ssq = nullptr;  // per-32 sums of squares of x [dim/32] (RMSNorm input)
  int32_t *token = nullptr, *pos = nullptr, *gen = nullptr;
  int32_t *fed = nullptr;             // token fed at each position [max_len]
  GbSampleParams *sample_p = nullptr; // device copy of the sampler parameters
  bool sampling = false;              // next/generate sample instead of argmax
  cudaGraphExec_t graph_sample = nullptr;
  // batched prefill workspace (allocated on first use): kPrefillChunk token rows
  float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr;
  __half *pf_a16 = nullptr, *pf_act16 = nullptr;
  int32_t *pf_tokens = nullptr;
  float *pf_part = nullptr;  // split-K partials of the prefill GEMMs
  float *pf_tmp = nullptr;   // tensor parallel: this rank's o / down partial [chunk][dim]
  size_t pf_part_floats = 0;
  AMap pf_map_dim, pf_map_q, pf_map_ffn;
  unsigned *err = nullptr;
  float *gemv_part = nullptr;
  unsigned *tile_counter = nullptr;
  float *attn_part = nullptr;
  unsigned *attn_counter = nullptr;
  unsigned long long *best = nullptr;
  // tensor parallel: peer exchange (receive buffers mapped by every rank)
  GbPeer peer;
  std::vector<void *> ipc_opened;  // peers' buffers and flags mapped into this process
  GbTagTable ttab = {};            // every rank's tagged partials (the o/down exchanges)
  unsigned *done = nullptr;
  int attn_splits = 1;
  GbGemvPlan plan_plain, plan_gu;
  cudaStream_t st = nullptr;
  cudaGraphExec_t graph = nullptr;
  ncclComm_t comm = nullptr;
  int32_t *h_stage = nullptr;  // pinned: token, pos, next, err
  float *h_logits = nullptr;   // pinned vocab floats
  std::vector<void *> allocs;
  int launches = 0;
  int sms = 148;
};

namespace {

// Every transfer and memset of a model goes on its own stream m->st: that
// stream is non-blocking, so work on the legacy default stream (a plain
// cudaMemset, which returns before a device-memory memset is done) would not
// be ordered before the uploads and kernels that follow on m->st.
template <class T>
int dalloc(gb_model *m, T **p, size_t n, const char *what) {
  void *q = nullptr;
  GB_CUDA(cudaMalloc(&q, n * sizeof(T) > 0 ? n * sizeof(T) : 16), what);
  GB_CUDA(cudaMemsetAsync(q, 0, n * sizeof(T) > 0 ? n * sizeof(T) : 16, m->st), what);
  m->allocs.push_back(q);
  *p = (T *)q;
  return GB_OK;
}

// Host decode of a norm-like tensor (model/model.go:186 norm(): quant.Dequantize).
int host_vector(const GbTensor *t, int n, std::vector<float> &out, const char *name) {
  if (!t) return gb_fail(GB_ERR_IO, "model: no tensor %s", name);
  if ((int)t->numel() != n)
    return gb_fail(GB_ERR_INVALID, "model: %s has %llu elements, want %d", name,
                   (unsigned long long)t->numel(), n);
  out.resize((size_t)n);
  switch (t->type) {
    case GB_T_F32: memcpy(out.data(), t->data, sizeof(float) * (size_t)n); break;
    case GB_T_F16:
      for (int i = 0; i < n; i++) out[i] = host_half((uint16_t)(t->data[2 * i] | t->data[2 * i + 1] << 8));
      break;
    case GB_T_BF16:
      for (int i = 0; i < n; i++) {
        uint32_t b = (uint32_t)(t->data[2 * i] | t->data[2 * i + 1] << 8) << 16;
        memcpy(&out[i], &b, 4);
      }
      break;
    default: return gb_fail(GB_ERR_UNSUPPORTED, "model: %s: %s norms not supported", name, tname(t->type));
  }
  return GB_OK;
}

int upload_vec(gb_model *m, const std::vector<float> &v, float **dst, const char *what) {
  int rc = dalloc(m, dst, v.size(), what);
  if (rc) return rc;
  GB_CUDA(cudaMemcpyAsync(*dst, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice, m->st), what);
  GB_CUDA(cudaStreamSynchronize(m->st), what);  // v is the caller's scratch
  return GB_OK;
}

// Host side of the uploads: two pinned buffers used in turn, so that the
// rows of the next chunk are gathered (by several host threads) while the
// previous chunk's copy to the device and its repack run on the stream.
struct Uploader {
  uint8_t *pin[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  size_t cap = 0;
  int cur = 0;
  int init(size_t bytes) {
    cap = bytes;
    for (int i = 0; i < 2; i++) {
      GB_CUDA(cudaMallocHost(&pin[i], cap), "model: pinned upload buffer");
      GB_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), "model: upload event");
    }
    return GB_OK;
  }
  ~Uploader() {
    for (int i = 0; i < 2; i++) {
      if (ev[i]) {
        cudaEventSynchronize(ev[i]);
        cudaEventDestroy(ev[i]);
      }
      if (pin[i]) cudaFreeHost(pin[i]);
    }
  }
};

// Gather n rows of sub_rb bytes (source stride rb) into dst with several threads.
void gather_rows(uint8_t *dst, const uint8_t *src, size_t rb, size_t sub_rb, int n) {
  const int nt = std::max(1, std::min(gb_host_threads(), (int)(((size_t)n * sub_rb) >> 22)));  // 4 MB a thread
  auto work = [&](int t) {
    for (int r = (int)((long long)n * t / nt); r < (int)((long long)n * (t + 1) / nt); r++)
      memcpy(dst + (size_t)r * sub_rb, src + (size_t)r * rb, sub_rb);
  };
  if (nt == 1) {
    work(0);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < nt; t++) th.emplace_back(work, t);
  for (auto &x : th) x.join();
}

// Upload rows [r0, r0+nr) and column super-blocks [c0, c0+nc) (in elements,
// multiples of 256) of a raw matrix into tiles [tile0, ...) of dst, in chunks
// of whole 32-row tiles that fit a pinned buffer. Stream-ordered: the caller
// synchronizes the stream before using the tiles.
int upload_tiles(const GbTensor *t, int r0, int nr, int c0, int nc, uint8_t *dst_base,
                 int dst_tile0, int dst_tile_mul, cudaStream_t st, uint8_t *staging,
                 size_t staging_bytes, Uploader *up) {
  const int typ = t->type;
  const size_t rb = (size_t)gb_row_bytes(typ, t->cols());
  const size_t sub_rb = (size_t)gb_row_bytes(typ, nc), coff = (size_t)gb_row_bytes(typ, c0);
  const int nsb = nc / 256;
  const size_t sbb = (size_t)gb_tiled_sb_bytes(typ);
  const int cr = std::max(32, (int)(up->cap / sub_rb) / 32 * 32);  // rows per chunk
  if ((size_t)cr * sub_rb > up->cap) return gb_fail(GB_ERR_INVALID, "model: pinned upload buffer too small");
  for (int i = 0; i < nr; i += cr) {
    const int n = std::min(cr, nr - i), ntiles = (n + 31) / 32, t0 = i / 32;
    const size_t need = sub_rb * (size_t)n;
    if (((need + 255) / 256) * 256 + (size_t)ntiles * nsb * sbb > staging_bytes)
      return gb_fail(GB_ERR_INVALID, "model: staging buffer too small");
    const int b = up->cur;
    GB_CUDA(cudaEventSynchronize(up->ev[b]), "model: upload");  // this buffer's previous copy is done
    gather_rows(up->pin[b], t->data + (size_t)(r0 + i) * rb + coff, rb, sub_rb, n);
    GB_CUDA(cudaMemcpyAsync(staging, up->pin[b], need, cudaMemcpyHostToDevice, st), "model: upload");
    GB_CUDA(cudaEventRecord(up->ev[b], st), "model: upload");
    up->cur ^= 1;
    if (dst_tile_mul == 1) {
      int rc = gb_repack_launch(typ, staging, n, nc, dst_base + ((size_t)dst_tile0 + t0) * nsb * sbb, st);
      if (rc) return rc;
    } else {
      // interleaved destination (gate/up pairs): repack into a scratch region
      // after the raw bytes, then place each sb-block at slot dst_tile0 of its
      // (row-block, super-block) pair, so that a gate/up unit is contiguous
      uint8_t *tmp = staging + ((need + 255) / 256) * 256;
      int rc = gb_repack_launch(typ, staging, n, nc, tmp, st);
      if (rc) return rc;
      GB_CUDA(cudaMemcpy2DAsync(dst_base + ((size_t)dst_tile0 + (size_t)dst_tile_mul * t0 * nsb) * sbb,
                                (size_t)dst_tile_mul * sbb, tmp, sbb, sbb, (size_t)ntiles * nsb,
                                cudaMemcpyDeviceToDevice, st),
              "model: place sb-blocks");
    }
  }
  return GB_OK;
}

// Tensor parallel: every rank allocates a buffer [slots][dim] of tagged
// 64-bit words for the partials of its row-split GEMVs (slots: o and down of
// every layer), a float buffer and flags [slots] for the lm_head's argmax key,
// exports them with CUDA IPC, gathers every rank's handles over NCCL (once,
// at load) and maps the peers' buffers, so that the step's kernels exchange
// partial sums with loads over NVLink instead of collectives.
int setup_peers(gb_model *m) {
  const gb_config &c = m->c;
  const int N = c.tp_world, R = c.tp_rank, slots = 2 * c.layers + 1;
  const int dim = std::max(c.dim, 2);
  float *buf = nullptr;
  unsigned *flag = nullptr, *epoch = nullptr;
  unsigned long long *tbuf = nullptr;
  int rc;
  if (N > kGbMaxWorld) return gb_fail(GB_ERR_UNSUPPORTED, "model: %d ranks (%d at most)", N, kGbMaxWorld);
  if ((rc = dalloc(m, &tbuf, (size_t)slots * dim, "model: peer buffers"))) return rc;
  if ((rc = dalloc(m, &buf, (size_t)slots * dim, "model: peer buffers")) ||
      (rc = dalloc(m, &flag, (size_t)slots, "model: peer flags")) || (rc = dalloc(m, &epoch, 1, "model: step counter")))
    return rc;
  struct Handles {
    cudaIpcMemHandle_t buf, flag, tbuf;
  } mine;
  GB_CUDA(cudaIpcGetMemHandle(&mine.tbuf, tbuf), "model: IPC handle");
  GB_CUDA(cudaIpcGetMemHandle(&mine.buf, buf), "model: IPC handle");
  GB_CUDA(cudaIpcGetMemHandle(&mine.flag, flag), "model: IPC handle");
  uint8_t *dh = nullptr;
  GB_CUDA(cudaMalloc(&dh, sizeof(Handles) * (size_t)(N + 1)), "model: IPC exchange");
  std::vector<Handles> all((size_t)N);
  cudaError_t e = cudaMemcpyAsync(dh + sizeof(Handles) * N, &mine, sizeof mine, cudaMemcpyHostToDevice, m->st);
  ncclResult_t nr = e == cudaSuccess ? nccl()->allGather(dh + sizeof(Handles) * N, dh, sizeof(Handles), ncclUint8,
                                                         m->comm, m->st)
                                     : ncclSuccess;
  if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(m->st);
  if (e == cudaSuccess && nr == ncclSuccess)
    e = cudaMemcpyAsync(all.data(), dh, sizeof(Handles) * N, cudaMemcpyDeviceToHost, m->st);
  if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(m->st);
  cudaFree(dh);
  if (nr != ncclSuccess) return gb_fail(GB_ERR_NCCL, "model: IPC exchange: %s", nccl()->getErrorString(nr));
  GB_CUDA(e, "model: IPC exchange");
  std::vector<float *> bufs((size_t)N);
  std::vector<unsigned *> flags((size_t)N);
  for (int q = 0; q < N; q++) {
    if (q == R) {
      bufs[q] = buf;
      flags[q] = flag;
      m->ttab.w[q] = tbuf;
      continue;
    }
    void *pb = nullptr, *pf = nullptr, *pt = nullptr;
    GB_CUDA(cudaIpcOpenMemHandle(&pt, all[q].tbuf, cudaIpcMemLazyEnablePeerAccess), "model: map peer buffer");
    m->ipc_opened.push_back(pt);
    m->ttab.w[q] = (const unsigned long long *)pt;
    GB_CUDA(cudaIpcOpenMemHandle(&pb, all[q].buf, cudaIpcMemLazyEnablePeerAccess), "model: map peer buffer");
    m->ipc_opened.push_back(pb);
    GB_CUDA(cudaIpcOpenMemHandle(&pf, all[q].flag, cudaIpcMemLazyEnablePeerAccess), "model: map peer flags");
    m->ipc_opened.push_back(pf);
    bufs[q] = (float *)pb;
    flags[q] = (unsigned *)pf;
  }
  float **dbufs = nullptr;
  unsigned **dflags = nullptr;
  if ((rc = dalloc(m, &dbufs, (size_t)N, "model: peer table")) || (rc = dalloc(m, &dflags, (size_t)N, "model: peer table")))
    return rc;
  GB_CUDA(cudaMemcpyAsync(dbufs, bufs.data(), sizeof(float *) * N, cudaMemcpyHostToDevice, m->st), "model: peer table");
  GB_CUDA(cudaMemcpyAsync(dflags, flags.data(), sizeof(unsigned *) * N, cudaMemcpyHostToDevice, m->st),
          "model: peer table");
  GB_CUDA(cudaStreamSynchronize(m->st), "model: peer table");
  GbPeer &P = m->peer;
  P.world = N;
  P.rank = R;
  P.dim = dim;
  P.bufs = dbufs;
  P.flags = dflags;
  P.my_buf = buf;
  P.my_flag = flag;
  P.my_tbuf = tbuf;
  P.epoch = epoch;
  return GB_OK;
}

int check_matrix(const GbGguf *f, const std::string &name, int rows, int cols, const GbTensor **out) {
  const GbTensor *t = f->tensor(name);
  if (!t) return gb_fail(GB_ERR_IO, "model: no tensor %s", name.c_str());
  if (t->dims.size() != 2) return gb_fail(GB_ERR_INVALID, "model: %s: not a matrix", name.c_str());
  if (t->rows() != rows || t->cols() != cols)
    return gb_fail(GB_ERR_INVALID, "model: %s is [%d][%d], want [%d][%d]", name.c_str(), t->rows(),
                   t->cols(), rows, cols);
  if (!gb_tiled_type(t->type))
    return gb_fail(GB_ERR_UNSUPPORTED, "model: %s: no kernel for %s weights", name.c_str(), tname(t->type));
  if (cols % 256)
    return gb_fail(GB_ERR_UNSUPPORTED, "model: %s: %d columns is not a multiple of 256", name.c_str(), cols);
  *out = t;
  return GB_OK;
}

int alloc_tiled(gb_model *m, Tiled *T, int ta, int tb, int split_tile, int ntiles, int nsb, int rows, int cols) {
  T->type_a = ta;
  T->type_b = tb;
  T->split_tile = split_tile;
  T->ntiles = ntiles;
  T->nsb = nsb;
  T->rows = rows;
  T->cols = cols;
  size_t na = (size_t)(split_tile < ntiles ? split_tile : ntiles) * nsb * gb_tiled_sb_bytes(ta);
  size_t nb = split_tile < ntiles ? (size_t)(ntiles - split_tile) * nsb * gb_tiled_sb_bytes(tb) : 0;
  T->bytes = na + nb;
  return dalloc(m, &T->w, T->bytes, "model: weights");
}

// ---- the decode step --------------------------------------------------------

struct Hook {
  cudaEvent_t ev[1024];
  int cls[1024];
  int n = 0;
};

// GEMV arguments; the input is x (float), RMS-normalised with `norm` in the
// GEMV's prologue when norm is non-null (per-32 sums of squares in m->ssq).
GbGemvArgs gemv_args(const Tiled &t, const float *x, const float *norm, float eps, int epi, gb_model *m) {
  GbGemvArgs a;
  a.w = t.w;
  a.type_a = t.type_a;
  a.type_b = t.type_b;
  a.split_tile = t.split_tile;
  a.rows = t.rows;
  a.ntiles = t.ntiles;
  a.nsb = t.nsb;
  a.in_x = x;
  a.in_w = norm;
  a.in_ssq = norm ? m->ssq : nullptr;
  a.eps = eps;
  a.epi = epi;
  a.e.err = m->err;
  a.e.part = m->gemv_part;
  a.e.tile_counter = m->tile_counter;
  a.e.pos = m->pos;
  a.e.max_len = m->c.max_len;
  return a;
}

int enqueue_step(gb_model *m, cudaStream_t st, Hook *hook, bool sample = false) {
  const gb_config &c = m->c;
  const bool pdl = true;
  const bool tp = c.tp_world > 1;
  int n = 0;
  auto mark = [&](int cls) -> int {
    n++;
    if (hook && hook->n < 1024) {
      hook->cls[hook->n] = cls;
      GB_CUDA(cudaEventRecord(hook->ev[hook->n], st), "model: profile event");
      hook->n++;
    }
    return GB_OK;
  };
  int rc;
  if (hook) {
    hook->cls[hook->n] = -1;
    GB_CUDA(cudaEventRecord(hook->ev[hook->n++], st), "model: profile event");
  }
  rc = gb_embed_launch(m->embd_type, m->embd.w, m->embd_nsb, c.dim, m->token, c.vocab, m->x, m->ssq,
                       m->err, m->fed, m->pos, c.max_len, st, pdl);
  if (rc || (rc = mark(K_OTHER))) return rc;
  for (int l = 0; l < c.layers; l++) {
    gb_model::Layer &L = m->layers[l];
    // attn RMSNorm in the prologue; q, k, v with RoPE and the KV-cache store in the epilogue
    GbGemvArgs a = gemv_args(L.qkv, m->x, L.attn_norm, c.eps, GB_EPI_QKV, m);
    a.e.q_out = m->q;
    a.e.kcache = L.kc;
    a.e.vcache = L.vc;
    a.e.q_rows = m->q_local;
    a.e.kv_rows = m->kv_local;
    a.e.head_dim = c.head_dim;
    a.e.kv_f16 = c.kv_f16;
    a.e.rope_cs = m->rope_cs;
    if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_QKV))) return rc;
    // attention over the cache
    GbAttnArgs at;
    at.q = m->q;
    at.k = L.kc;
    at.v = L.vc;
    at.kv_f16 = c.kv_f16;
    const int V = c.kv_f16 ? 8 : 4;
    at.k_sh = (long long)c.head_dim * c.max_len;
    at.k_sd = (long long)c.max_len * V;
    at.k_st = V;
    at.v_sh = (long long)c.max_len * c.head_dim;
    at.v_st = c.kv_f16 ? V : c.head_dim;  // fp16 V is stored in the K layout
    at.v_sd = c.kv_f16 ? (long long)c.max_len * V : 0;
    at.n_heads = m->q_local / c.head_dim;
    at.n_kv = m->kv_local / c.head_dim;
    at.head_dim = c.head_dim;
    at.scale = (float)(1 / sqrt((double)c.head_dim));  // model/model.go:322
    at.kv_len_pos = m->pos;
    at.max_len = c.max_len;
    at.splits = m->attn_splits;
    at.out = m->attn;
    at.part = m->attn_part;
    at.counter = m->attn_counter;
    at.err = m->err;
    if (L.tmap) {
      at.tmap = 1;
      at.tk = L.tk;
      at.tv = L.tv;
    }
    if ((rc = gb_attn_launch(at, st, pdl)) || (rc = mark(K_ATTN))) return rc;
    // o projection + residual (+ sums of squares for the FFN norm)
    if (!tp) {
      a = gemv_args(L.wo, m->attn, nullptr, c.eps, GB_EPI_RESID, m);
      a.e.x = m->x;
      a.e.ssq = m->ssq;
      if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_O))) return rc;
    } else {
      // partials to every rank's peer slot 2l; sum + residual once all arrived
      a = gemv_args(L.wo, m->attn, nullptr, c.eps, GB_EPI_PARTIAL, m);
      a.e.peer = m->peer;
      a.e.peer_slot = 2 * l;
      if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_O))) return rc;
      if ((rc = gb_peer_resid_tagged_launch(m->ttab, c.tp_world, m->peer.epoch, m->peer.wait_limit, 2 * l,
                                            m->peer.dim, m->x, c.dim, m->ssq, m->err, st, pdl)) ||
          (rc = mark(K_OTHER)))
        return rc;
    }
    // FFN RMSNorm in the prologue; gate/up + SwiGLU
    a = gemv_args(L.gu, m->x, L.ffn_norm, c.eps, GB_EPI_SWIGLU, m);
    a.e.y = m->act;
    if ((rc = gb_gemv_launch(a, m->plan_gu, st, pdl)) || (rc = mark(K_GU))) return rc;
    // down + residual (+ sums of squares for the next norm)
    if (!tp) {
      a = gemv_args(L.down, m->act, nullptr, c.eps, GB_EPI_RESID, m);
      a.e.x = m->x;
      a.e.ssq = m->ssq;
      if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_DOWN))) return rc;
    } else {
      a = gemv_args(L.down, m->act, nullptr, c.eps, GB_EPI_PARTIAL, m);
      a.e.peer = m->peer;
      a.e.peer_slot = 2 * l + 1;
      if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_DOWN))) return rc;
      if ((rc = gb_peer_resid_tagged_launch(m->ttab, c.tp_world, m->peer.epoch, m->peer.wait_limit, 2 * l + 1,
                                            m->peer.dim, m->x, c.dim, m->ssq, m->err, st, pdl)) ||
          (rc = mark(K_OTHER)))
        return rc;
    }
  }
  // output RMSNorm in the prologue; lm_head + argmax (model.Argmax on the device)
  GbGemvArgs a = gemv_args(m->head, m->x, m->out_norm, c.eps, GB_EPI_LOGITS, m);
  a.e.y = m->logits;
  a.e.best = m->best;
  a.e.counter = m->done;
  a.e.row_offset = m->vocab_off;
  a.e.vocab_total = c.vocab;
  if (!tp) {
    a.e.token_out = m->token;
    a.e.token_hist = m->gen;
  } else {
    a.e.peer = m->peer;  // the local argmax key goes to every rank's slot 2L
    a.e.peer_slot = 2 * c.layers;
  }
  if ((rc = gb_gemv_launch(a, m->plan_plain, st, pdl)) || (rc = mark(K_HEAD))) return rc;
  if (tp && ((rc = gb_peer_argmax_launch(m->peer, 2 * c.layers, m->token, m->gen, m->pos, c.max_len, m->err, st,
                                         pdl)) ||
             (rc = mark(K_OTHER))))
    return rc;
  // the sampler replaces the argmax token (and its history slot) of the head's epilogue
  if (sample && ((rc = gb_sample_launch(m->logits, c.vocab, nullptr, m->sample_p, nullptr, 0, m->fed, m->pos,
                                        c.max_len, 0, m->token, m->gen, m->err, st)) ||
                 (rc = mark(K_OTHER))))
    return rc;
  if ((rc = gb_advance_pos_launch(m->pos, tp ? (unsigned *)m->peer.epoch : nullptr, st)) || (rc = mark(K_OTHER)))
    return rc;
  m->launches = n;
  return GB_OK;
}

int capture(gb_model *m, bool sample = false) {
  cudaGraph_t g = nullptr;
  GB_CUDA(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal), "model: graph capture");
  const int launches = m->launches;
  int rc = enqueue_step(m, m->st, nullptr, sample);
  if (sample) m->launches = launches;  // the greedy step's count stays the model's figure
  cudaError_t e = cudaStreamEndCapture(m->st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return gb_cuda_fail(e, "model: graph capture");
  e = cudaGraphInstantiate(sample ? &m->graph_sample : &m->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return gb_cuda_fail(e, "model: graph instantiate");
  return GB_OK;
}

// One step with the model's token rule (argmax, or the sampler when set).
int run_step(gb_model *m) {
  if (m->sampling) {
    if (m->graph_sample) {
      GB_CUDA(cudaGraphLaunch(m->graph_sample, m->st), "model: graph launch");
      return GB_OK;
    }
    const int launches = m->launches;
    int rc = enqueue_step(m, m->st, nullptr, true);
    m->launches = launches;
    return rc;
  }
  if (m->graph) {
    GB_CUDA(cudaGraphLaunch(m->graph, m->st), "model: graph launch");
    return GB_OK;
  }
  return enqueue_step(m, m->st, nullptr);
}

// forward() returns logits: the argmax step is enough (same logits).
int run_logits_step(gb_model *m) {
  const bool s = m->sampling;
  m->sampling = false;
  int rc = run_step(m);
  m->sampling = s;
  return rc;
}

int check_err(gb_model *m) {
  GB_CUDA(cudaMemcpyAsync(m->h_stage + 3, m->err, sizeof(unsigned), cudaMemcpyDeviceToHost, m->st),
          "model: status");
  GB_CUDA(cudaStreamSynchronize(m->st), "model: forward");
  unsigned e = (unsigned)m->h_stage[3];
  if (e) {
    GB_CUDA(cudaMemsetAsync(m->err, 0, sizeof(unsigned), m->st), "model: status");
    GB_CUDA(cudaStreamSynchronize(m->st), "model: status");
    if (e & GB_DEVERR_TIMEOUT) return gb_fail(GB_ERR_TIMEOUT, "model: a bounded device wait timed out");
    if (e & GB_DEVERR_POS) return gb_fail(GB_ERR_DEVICE, "model: position outside the KV cache");
    return gb_fail(GB_ERR_DEVICE, "model: token outside the vocabulary");
  }
  return GB_OK;
}

int set_token_pos(gb_model *m, int32_t token, int pos) {
  // model/model.go:315-320
  if (pos < 0 || pos >= m->c.max_len)
    return gb_fail(GB_ERR_INVALID, "model: position %d outside the %d-token cache", pos, m->c.max_len);
  if (token < 0 || token >= m->c.vocab)
    return gb_fail(GB_ERR_INVALID, "model: token %d outside the vocabulary", token);
  m->h_stage[0] = token;
  m->h_stage[1] = pos;
  GB_CUDA(cudaMemcpyAsync(m->token, m->h_stage, sizeof(int32_t), cudaMemcpyHostToDevice, m->st), "model: token");
  GB_CUDA(cudaMemcpyAsync(m->pos, m->h_stage + 1, sizeof(int32_t), cudaMemcpyHostToDevice, m->st), "model: position");
  return GB_OK;
}

void free_model(gb_model *m) {
  if (!m) return;
  if (m->graph) cudaGraphExecDestroy(m->graph);
  if (m->graph_sample) cudaGraphExecDestroy(m->graph_sample);
  for (void *p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  if (m->comm && nccl() && nccl()->commDestroy) nccl()->commDestroy(m->comm);
  for (void *p : m->allocs) cudaFree(p);
  if (m->h_stage) cudaFreeHost(m->h_stage);
  if (m->h_logits) cudaFreeHost(m->h_logits);
  if (m->st) cudaStreamDestroy(m->st);
  delete m;
}

int load_model(GbGguf *f, const gb_model_opts *opts, gb_model **out) {
  gb_model_opts o;
  gb_model_opts_default(&o);
  if (opts) o = *opts;
  // model/model.go:35 ConfigFrom
  std::string arch = f->get_string("general.architecture", "");
  if (arch != "llama") return gb_fail(GB_ERR_INVALID, "model: architecture \"%s\" is not llama", arch.c_str());
  gb_config c{};
  c.layers = (int)f->get_uint("llama.block_count", 0);
  c.dim = (int)f->get_uint("llama.embedding_length", 0);
  c.ffn = (int)f->get_uint("llama.feed_forward_length", 0);
  c.heads = (int)f->get_uint("llama.attention.head_count", 0);
  c.ctx_len = (int)f->get_uint("llama.context_length", 2048);
  c.rope_base = (float)f->get_float("llama.rope.freq_base", 10000);
  c.eps = (float)f->get_float("llama.attention.layer_norm_rms_epsilon", 1e-5);
  c.kv_heads = (int)f->get_uint("llama.attention.head_count_kv", (uint64_t)c.heads);
  if (c.layers == 0 || c.dim == 0 || c.ffn == 0 || c.heads == 0)
    return gb_fail(GB_ERR_INVALID, "model: incomplete llama metadata");
  c.head_dim = (int)f->get_uint("llama.attention.key_length", (uint64_t)(c.dim / c.heads));
  if (c.kv_heads == 0 || c.heads % c.kv_heads != 0)
    return gb_fail(GB_ERR_INVALID, "model: %d heads is not a multiple of %d KV heads", c.heads, c.kv_heads);
  const GbTensor *embd = f->tensor("token_embd.weight");
  if (!embd) return gb_fail(GB_ERR_IO, "model: no token_embd.weight");
  if (embd->dims.size() != 2 || embd->cols() != c.dim)
    return gb_fail(GB_ERR_INVALID, "model: token_embd.weight is not [vocab][%d]", c.dim);
  c.vocab = embd->rows();
  // model/model.go:165: maxLen <= 0 or beyond the trained context -> context length
  c.max_len = (o.max_len <= 0 || o.max_len > c.ctx_len) ? c.ctx_len : o.max_len;
  c.kv_f16 = o.kv_f16 ? 1 : 0;
  c.tp_rank = o.tp_rank;
  c.tp_world = o.tp_world < 1 ? 1 : o.tp_world;
  const int N = c.tp_world, R = c.tp_rank;
  if (R < 0 || R >= N) return gb_fail(GB_ERR_INVALID, "model: rank %d outside world %d", R, N);
  if (c.head_dim != 64 && c.head_dim != 128)
    return gb_fail(GB_ERR_UNSUPPORTED, "model: head_dim %d (64 or 128 supported)", c.head_dim);
  if (c.heads % N || c.kv_heads % N || c.ffn % (256 * N) || (c.heads / N * c.head_dim) % 256 ||
      c.vocab % N || c.dim % 256)
    return gb_fail(GB_ERR_UNSUPPORTED, "model: shape does not split over %d GPUs", N);
  if (N > 1 && !nccl()) return gb_fail(GB_ERR_NCCL, "model: libnccl.so.2 not found");

  gb_model *m = new gb_model();
  m->c = c;
  m->o = o;
  int rc = GB_OK;
  auto fail = [&](int r) {
    free_model(m);
    return r;
  };
  if (cudaSetDevice(o.device) != cudaSuccess) return fail(gb_fail(GB_ERR_CUDA, "model: no device %d", o.device));
  cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, o.device);
  if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess)
    return fail(gb_fail(GB_ERR_CUDA, "model: stream"));
  const int hd = c.head_dim, kv_dim = c.kv_heads * hd;
  m->q_local = c.heads / N * hd;
  m->kv_local = c.kv_heads / N * hd;
  m->ffn_local = c.ffn / N;
  m->vocab_local = c.vocab / N;
  m->vocab_off = R * m->vocab_local;
  (void)kv_dim;

  // staging for uploads: the largest raw shard plus its tiled copy
  size_t staging_bytes = 0;
  for (auto &t : f->tensors) staging_bytes = std::max<size_t>(staging_bytes, (size_t)t.bytes);
  staging_bytes = staging_bytes * 2 + (1 << 20);
  uint8_t *staging = nullptr;
  if ((rc = dalloc(m, &staging, staging_bytes, "model: staging"))) return fail(rc);
  // pinned host chunks: 32 MB, at least one 32-row tile of the widest row
  size_t widest = 0;
  for (auto &t : f->tensors)
    if (t.cols() > 0) widest = std::max<size_t>(widest, (size_t)gb_row_bytes(t.type, t.cols()));
  Uploader up;
  if ((rc = up.init(std::max<size_t>((size_t)32 << 20, 32 * widest)))) return fail(rc);

  // token embedding (full, for the lookup) -- tiled
  if (!gb_tiled_type(embd->type))
    return fail(gb_fail(GB_ERR_UNSUPPORTED, "model: token_embd.weight: no kernel for %s", tname(embd->type)));
  m->embd_type = embd->type;
  m->embd_nsb = c.dim / 256;
  {
    int nt = (c.vocab + 31) / 32;
    if ((rc = alloc_tiled(m, &m->embd, embd->type, embd->type, 1 << 30, nt, c.dim / 256, c.vocab, c.dim)))
      return fail(rc);
    // upload in row chunks to bound the staging size
    int chunk = (int)std::max<size_t>(32, (staging_bytes / 2 / (size_t)gb_row_bytes(embd->type, c.dim)) / 32 * 32);
    for (int r0 = 0; r0 < c.vocab; r0 += chunk) {
      int nr = std::min(chunk, c.vocab - r0);
      if ((rc = upload_tiles(embd, r0, nr, 0, c.dim, m->embd.w, r0 / 32, 1, m->st, staging, staging_bytes, &up)))
        return fail(rc);
    }
  }

  m->layers.resize((size_t)c.layers);
  std::vector<float> hv;
  for (int l = 0; l < c.layers; l++) {
    gb_model::Layer &L = m->layers[(size_t)l];
    std::string p = "blk." + std::to_string(l) + ".";
    if ((rc = host_vector(f->tensor(p + "attn_norm.weight"), c.dim, hv, (p + "attn_norm.weight").c_str())) ||
        (rc = upload_vec(m, hv, &L.attn_norm, "model: norm")))
      return fail(rc);
    if ((rc = host_vector(f->tensor(p + "ffn_norm.weight"), c.dim, hv, (p + "ffn_norm.weight").c_str())) ||
        (rc = upload_vec(m, hv, &L.ffn_norm, "model: norm")))
      return fail(rc);
    const GbTensor *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    if ((rc = check_matrix(f, p + "attn_q.weight", c.heads * hd, c.dim, &wq)) ||
        (rc = check_matrix(f, p + "attn_k.weight", c.kv_heads * hd, c.dim, &wk)) ||
        (rc = check_matrix(f, p + "attn_v.weight", c.kv_heads * hd, c.dim, &wv)) ||
        (rc = check_matrix(f, p + "attn_output.weight", c.dim, c.heads * hd, &wo)) ||
        (rc = check_matrix(f, p + "ffn_gate.weight", c.ffn, c.dim, &wg)) ||
        (rc = check_matrix(f, p + "ffn_up.weight", c.ffn, c.dim, &wu)) ||
        (rc = check_matrix(f, p + "ffn_down.weight", c.dim, c.ffn, &wd)))
      return fail(rc);
    if (wq->type != wk->type)
      return fail(gb_fail(GB_ERR_UNSUPPORTED, "model: %sattn_q and attn_k types differ", p.c_str()));
    if (wg->type != wu->type)
      return fail(gb_fail(GB_ERR_UNSUPPORTED, "model: %sffn_gate and ffn_up types differ", p.c_str()));
    // q | k | v rows of this rank, one tiled buffer (q,k type_a; v type_b)
    const int tq = m->q_local / 32, tk = m->kv_local / 32, tv = m->kv_local / 32;
    if ((rc = alloc_tiled(m, &L.qkv, wq->type, wv->type, wv->type == wq->type ? (1 << 30) : tq + tk,
                          tq + tk + tv, c.dim / 256, m->q_local + 2 * m->kv_local, c.dim)))
      return fail(rc);
    const size_t sba = (size_t)gb_tiled_sb_bytes(wq->type) * (c.dim / 256);
    if ((rc = upload_tiles(wq, R * m->q_local, m->q_local, 0, c.dim, L.qkv.w, 0, 1, m->st, staging, staging_bytes, &up)) ||
        (rc = upload_tiles(wk, R * m->kv_local, m->kv_local, 0, c.dim, L.qkv.w, tq, 1, m->st, staging, staging_bytes, &up)) ||
        (rc = upload_tiles(wv, R * m->kv_local, m->kv_local, 0, c.dim, L.qkv.w + (size_t)(tq + tk) * sba, 0, 1,
                           m->st, staging, staging_bytes, &up)))
      return fail(rc);
    // o: all dim rows, this rank's input columns
    if ((rc = alloc_tiled(m, &L.wo, wo->type, wo->type, 1 << 30, c.dim / 32, m->q_local / 256, c.dim, m->q_local)) ||
        (rc = upload_tiles(wo, 0, c.dim, R * m->q_local, m->q_local, L.wo.w, 0, 1, m->st, staging, staging_bytes, &up)))
      return fail(rc);
    // gate/up: this rank's FFN rows; per (row-block, super-block) the gate then the up sb-block
    const int tf = m->ffn_local / 32;
    if ((rc = alloc_tiled(m, &L.gu, wg->type, wg->type, 1 << 30, 2 * tf, c.dim / 256, 2 * m->ffn_local, c.dim)) ||
        (rc = upload_tiles(wg, R * m->ffn_local, m->ffn_local, 0, c.dim, L.gu.w, 0, 2, m->st, staging, staging_bytes, &up)) ||
        (rc = upload_tiles(wu, R * m->ffn_local, m->ffn_local, 0, c.dim, L.gu.w, 1, 2, m->st, staging, staging_bytes, &up)))
      return fail(rc);
    // down: all dim rows, this rank's FFN columns
    if ((rc = alloc_tiled(m, &L.down, wd->type, wd->type, 1 << 30, c.dim / 32, m->ffn_local / 256, c.dim, m->ffn_local)) ||
        (rc = upload_tiles(wd, 0, c.dim, R * m->ffn_local, m->ffn_local, L.down.w, 0, 1, m->st, staging, staging_bytes, &up)))
      return fail(rc);
    // KV caches, head-major (see gb_attn.cu)
    const size_t elems = (size_t)(m->kv_local) * c.max_len;
    const size_t esz = c.kv_f16 ? 2 : 4;
    uint8_t *kc = nullptr, *vc = nullptr;
    if ((rc = dalloc(m, &kc, elems * esz, "model: KV cache")) || (rc = dalloc(m, &vc, elems * esz, "model: KV cache")))
      return fail(rc);
    L.kc = kc;
    L.vc = vc;
    if (c.kv_f16) {  // whole 128-position sub-chunks then move with one TMA copy each
      L.tmap = gb_attn_tensor_maps(kc, vc, m->kv_local / hd, hd, c.max_len, &L.tk, &L.tv) == GB_OK;
      if (!L.tmap) gb_clear_error();
    }
  }
  if ((rc = host_vector(f->tensor("output_norm.weight"), c.dim, hv, "output_norm.weight")) ||
      (rc = upload_vec(m, hv, &m->out_norm, "model: norm")))
    return fail(rc);
  // lm_head: output.weight, or tied to token_embd (model/model.go:263-267)
  const GbTensor *head = f->tensor("output.weight");
  if (head) {
    const GbTensor *h2;
    rc = check_matrix(f, "output.weight", c.vocab, c.dim, &h2);
    if (rc) return fail(rc);
    if ((rc = alloc_tiled(m, &m->head, head->type, head->type, 1 << 30, (m->vocab_local + 31) / 32, c.dim / 256,
                          m->vocab_local, c.dim)))
      return fail(rc);
    int chunk = (int)std::max<size_t>(32, (staging_bytes / 2 / (size_t)gb_row_bytes(head->type, c.dim)) / 32 * 32);
    for (int r0 = 0; r0 < m->vocab_local; r0 += chunk) {
      int nr = std::min(chunk, m->vocab_local - r0);
      if ((rc = upload_tiles(head, m->vocab_off + r0, nr, 0, c.dim, m->head.w, r0 / 32, 1, m->st, staging,
                             staging_bytes, &up)))
        return fail(rc);
    }
  } else {
    if (m->vocab_off % 32 || (N > 1 && m->vocab_local % 32))
      return fail(gb_fail(GB_ERR_UNSUPPORTED, "model: tied head shard is not tile aligned"));
    m->head = m->embd;
    m->head.owned = false;
    m->head.w = m->embd.w + (size_t)(m->vocab_off / 32) * m->embd.nsb * gb_tiled_sb_bytes(m->embd.type_a);
    m->head.rows = m->vocab_local;
    m->head.ntiles = (m->vocab_local + 31) / 32;
  }
  // RoPE angles (cpu.RoPE, backend/cpu/cpu.go:69) in float64 on the host
  {
    std::vector<float> freq((size_t)hd / 2, 1.f);
    bool has_freq = false;
    if (const GbTensor *ft = f->tensor("rope_freqs.weight")) {
      if ((rc = host_vector(ft, hd / 2, freq, "rope_freqs.weight"))) return fail(rc);
      has_freq = true;
    }
    std::vector<double> cs((size_t)c.max_len * (hd / 2) * 2);
    for (int p = 0; p < c.max_len; p++)
      for (int j = 0; j < hd / 2; j++) {
        double theta = (double)p * pow((double)c.rope_base, -2 * (double)j / (double)hd);
        if (has_freq) theta /= (double)freq[(size_t)j];
        cs[((size_t)p * (hd / 2) + j) * 2] = cos(theta);
        cs[((size_t)p * (hd / 2) + j) * 2 + 1] = sin(theta);
      }
    if ((rc = dalloc(m, &m->rope_cs, cs.size(), "model: rope table"))) return fail(rc);
    if (cudaMemcpyAsync(m->rope_cs, cs.data(), cs.size() * sizeof(double), cudaMemcpyHostToDevice, m->st) !=
            cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess)
      return fail(gb_fail(GB_ERR_CUDA, "model: rope table upload"));
  }
  // work buffers
  if ((rc = dalloc(m, &m->x, (size_t)c.dim, "model: work")) || (rc = dalloc(m, &m->q, (size_t)m->q_local, "model: work")) ||
      (rc = dalloc(m, &m->attn, (size_t)m->q_local, "model: work")) ||
      (rc = dalloc(m, &m->logits, (size_t)m->vocab_local, "model: work")) ||
      (rc = dalloc(m, &m->logits_full, (size_t)c.vocab, "model: work")) ||
      (rc = dalloc(m, &m->token, 4, "model: work")) || (rc = dalloc(m, &m->pos, 4, "model: work")) ||
      (rc = dalloc(m, &m->gen, (size_t)c.max_len, "model: work")) || (rc = dalloc(m, &m->err, 4, "model: work")) ||
      (rc = dalloc(m, &m->fed, (size_t)c.max_len, "model: work")) ||
      (rc = dalloc(m, &m->sample_p, 1, "model: work")) ||
      (rc = dalloc(m, &m->best, 1, "model: work")) || (rc = dalloc(m, &m->done, 1, "model: work")))
    return fail(rc);
  if ((rc = dalloc(m, &m->act, (size_t)m->ffn_local, "model: work")) ||
      (rc = dalloc(m, &m->ssq, (size_t)c.dim / 32, "model: work")))
    return fail(rc);
  m->plan_plain = gb_gemv_plan(0, 0, GB_EPI_PLAIN, m->sms);
  m->plan_gu = gb_gemv_plan(0, 0, GB_EPI_SWIGLU, m->sms);
  int max_tiles = std::max(std::max(m->head.ntiles, (m->q_local + 2 * m->kv_local) / 32),
                           std::max(c.dim / 32, 2 * m->ffn_local / 32));
  if ((rc = dalloc(m, &m->gemv_part, (size_t)gb_gemv_scratch_floats(0, m->plan_plain), "model: scratch")) ||
      (rc = dalloc(m, &m->tile_counter, (size_t)max_tiles + 64, "model: scratch")))
    return fail(rc);
  m->attn_splits = gb_attn_splits(m->kv_local / hd, c.max_len, m->sms);
  if ((rc = dalloc(m, &m->attn_part,
                   gb_attn_part_floats(m->kv_local / hd, m->attn_splits, c.heads / c.kv_heads, hd), "model: scratch")) ||
      (rc = dalloc(m, &m->attn_counter, (size_t)(m->kv_local / hd), "model: scratch")))
    return fail(rc);
  if (cudaMallocHost(&m->h_stage, 64) != cudaSuccess || cudaMallocHost(&m->h_logits, sizeof(float) * (size_t)c.vocab) != cudaSuccess)
    return fail(gb_fail(GB_ERR_CUDA, "model: pinned host buffers"));
  // the staging buffer is no longer needed
  cudaFree(staging);
  m->allocs.erase(std::find(m->allocs.begin(), m->allocs.end(), (void *)staging));
  if (N > 1) {
    if (!o.nccl_id) return fail(gb_fail(GB_ERR_INVALID, "model: tp_world %d needs an NCCL id", N));
    ncclUniqueId id;
    memcpy(&id, o.nccl_id, sizeof id);
    ncclResult_t r = nccl()->commInitRank(&m->comm, N, id, R);
    if (r != ncclSuccess) return fail(gb_fail(GB_ERR_NCCL, "model: NCCL init: %s", nccl()->getErrorString(r)));
    if ((rc = setup_peers(m))) return fail(rc);
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(gb_fail(GB_ERR_CUDA, "model: load"));
  // embedding, 5 per layer (+2 per layer for the collectives' residual
  // kernels under tensor parallelism), lm_head, (+key reduce), advance
  m->launches = 1 + c.layers * (5 + (N > 1 ? 2 : 0)) + 1 + (N > 1 ? 1 : 0) + 1;
  if (o.use_graph && (rc = capture(m))) return fail(rc);
  *out = m;
  return GB_OK;
}

}  // namespace

namespace {

constexpr int kPrefillChunk = 512;  // token rows per batched pass (4 M-tiles of the GEMM)

int prefill_workspace(gb_model *m) {
  if (m->pf_x) return GB_OK;
  const gb_config &c = m->c;
  const int Tc = kPrefillChunk, qkv = m->q_local + 2 * m->kv_local;
  const size_t a16 = (size_t)Tc * std::max(c.dim, m->q_local);
  int rc;
  if ((rc = dalloc(m, &m->pf_x, (size_t)Tc * c.dim, "model: prefill workspace")) ||
      (rc = dalloc(m, &m->pf_qkv, (size_t)Tc * qkv, "model: prefill workspace")) ||
      (rc = dalloc(m, &m->pf_q, (size_t)Tc * m->q_local, "model: prefill workspace")) ||
      (rc = dalloc(m, &m->pf_a16, a16, "model: prefill workspace")) ||
      (rc = dalloc(m, &m->pf_act16, (size_t)Tc * m->ffn_local, "model: prefill workspace")) ||
      (rc = dalloc(m, &m->pf_tokens, (size_t)Tc, "model: prefill workspace")))
    return rc;
  // split-K partials: a plan never has more CTAs with partials than SMs, each
  // at most 4 token tiles x 128 columns (or 2 x 256 for the gate/up pairs)
  m->pf_part_floats = (size_t)m->sms * 4 * 128 * 128;
  if ((rc = dalloc(m, &m->pf_part, m->pf_part_floats, "model: prefill workspace"))) return rc;
  if (c.tp_world > 1 && (rc = dalloc(m, &m->pf_tmp, (size_t)Tc * c.dim, "model: prefill workspace"))) return rc;
  for (int box : {128, 16}) {
    const auto pick = [box](AMap &a) { return box == 128 ? &a.a128 : &a.a16; };
    if ((rc = gb_tmap_f16_rows(m->pf_a16, Tc, c.dim, pick(m->pf_map_dim), box)) ||
        (rc = gb_tmap_f16_rows(m->pf_a16, Tc, m->q_local, pick(m->pf_map_q), box)) ||
        (rc = gb_tmap_f16_rows(m->pf_act16, Tc, m->ffn_local, pick(m->pf_map_ffn), box)))
      return rc;
  }
  return GB_OK;
}

GbTcGemm tc_args(const Tiled &t, int epi, int T, const AMap &map, gb_model *m) {
  GbTcGemm g;
  g.w = t.w;
  g.type_a = t.type_a;
  g.type_b = t.type_b;
  g.split_tile = t.split_tile;
  g.rows = t.rows;
  g.ntiles = t.ntiles;
  g.nsb = t.nsb;
  g.epi = epi;
  g.T = T;
  g.err = m->err;
  g.part = m->pf_part;
  g.part_floats = m->pf_part_floats;
  g.tmap_a = map.a128;
  g.tmap_a16 = map.a16;
  g.a16 = true;
  if (t.w16) {
    g.w16 = t.w16;
    g.tmap_b = t.map16;
  }
  return g;
}

// x += A W^T for the row-parallel o and down projections. Under tensor
// parallelism each rank's product over its input columns is a partial: the
// ranks' partials are summed by an NCCL all-reduce on the model stream (every
// rank makes the same calls in the same order), then added to x.
int row_parallel(gb_model *m, const Tiled &w, int T, const AMap &map) {
  const gb_config &c = m->c;
  const bool tp = c.tp_world > 1;
  GbTcGemm g = tc_args(w, tp ? GB_EPI_PLAIN : GB_EPI_RESID, T, map, m);
  g.y = tp ? m->pf_tmp : m->pf_x;
  g.ldy = c.dim;
  int rc = gb_tc_gemm_launch(g, m->st);
  if (rc || !tp) return rc;
  GB_NCCL(nccl()->allReduce(m->pf_tmp, m->pf_tmp, (size_t)T * c.dim, ncclFloat, ncclSum, m->comm, m->st),
          "model: prefill all-reduce");
  return gb_add_launch(m->pf_x, m->pf_tmp, m->pf_x, T * c.dim, m->st);
}

// Tokens [0, T) of one chunk at positions p0..: every layer's K/V; the
// residual stream of the last layer is not needed (the next step reads only
// the cache), so that layer stops after its K/V.
int prefill_chunk(gb_model *m, int T, int p0) {
  const gb_config &c = m->c;
  cudaStream_t st = m->st;
  const int hd = c.head_dim, qkv = m->q_local + 2 * m->kv_local;
  int rc = gb_embed_rows_launch(m->embd_type, m->embd.w, m->embd_nsb, c.dim, m->pf_tokens, T, c.vocab, m->pf_x,
                                m->fed, p0, c.max_len, m->err, st);
  if (rc) return rc;
  for (int l = 0; l < c.layers; l++) {
    gb_model::Layer &L = m->layers[(size_t)l];
    if ((rc = gb_rmsnorm_rows_f16_launch(m->pf_x, L.attn_norm, T, c.dim, c.eps, m->pf_a16, st))) return rc;
    GbTcGemm g = tc_args(L.qkv, GB_EPI_PLAIN, T, m->pf_map_dim, m);
    g.y = m->pf_qkv;
    g.ldy = qkv;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
    if ((rc = gb_rope_kv_launch(m->pf_qkv, T, m->q_local, m->kv_local, hd, m->rope_cs, p0, c.max_len, c.kv_f16,
                                m->pf_q, L.kc, L.vc, st)))
      return rc;
    if (l == c.layers - 1) break;
    if ((rc = gb_attn_prefill_launch(m->pf_q, T, p0, m->q_local / hd, m->kv_local / hd, hd, L.kc, L.vc, c.kv_f16,
                                     c.max_len, m->pf_a16, st)))
      return rc;
    if ((rc = row_parallel(m, L.wo, T, m->pf_map_q))) return rc;
    if ((rc = gb_rmsnorm_rows_f16_launch(m->pf_x, L.ffn_norm, T, c.dim, c.eps, m->pf_a16, st))) return rc;
    g = tc_args(L.gu, GB_EPI_SWIGLU, T, m->pf_map_dim, m);
    g.rows = m->ffn_local;  // one half of the gate/up pairs
    g.ntiles = L.gu.ntiles / 2;
    g.act = m->pf_act16;
    g.ld_act = m->ffn_local;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
    if ((rc = row_parallel(m, L.down, T, m->pf_map_ffn))) return rc;
  }
  return GB_OK;
}

}  // namespace

// ---- C ABI: model -------------------------------------------------------------
extern "C" {

void gb_model_opts_default(gb_model_opts *o) {
  memset(o, 0, sizeof *o);
  o->device = 0;
  o->max_len = 0;
  o->kv_f16 = 1;
  o->use_graph = 1;
  o->tp_rank = 0;
  o->tp_world = 1;
}

int gb_model_load(const char *path, const gb_model_opts *opts, gb_model **out) {
  gb_clear_error();
  if (!path || !out) return gb_fail(GB_ERR_INVALID, "model: null argument");
  std::unique_ptr<GbGguf> f(gb_gguf_open(path));
  if (!f) return GB_ERR_IO;
  return load_model(f.get(), opts, out);
}

int gb_model_load_mem(const void *gguf, size_t len, const gb_model_opts *opts, gb_model **out) {
  gb_clear_error();
  if (!gguf || !out) return gb_fail(GB_ERR_INVALID, "model: null argument");
  std::unique_ptr<GbGguf> f(gb_gguf_parse((const uint8_t *)gguf, len));
  if (!f) return GB_ERR_IO;
  return load_model(f.get(), opts, out);
}

int gb_model_config(const gb_model *m, gb_config *c) {
  gb_clear_error();
  if (!m || !c) return gb_fail(GB_ERR_INVALID, "model: null argument");
  *c = m->c;
  return GB_OK;
}

int gb_model_forward(gb_model *m, int32_t token, int pos, float *host_logits) {
  gb_clear_error();
  if (!m) return gb_fail(GB_ERR_INVALID, "model: null model");
  int rc = set_token_pos(m, token, pos);
  if (rc || (rc = run_logits_step(m))) return rc;
  const float *src = m->logits;
  if (m->c.tp_world > 1) {
    GB_NCCL(nccl()->allGather(m->logits, m->logits_full, (size_t)m->vocab_local, ncclFloat, m->comm, m->st),
            "model: logits all-gather");
    src = m->logits_full;
  }
  // a page-locked caller buffer takes the copy directly; pageable memory goes
  // through the model's pinned staging buffer and one host copy
  bool pinned = false;
  if (host_logits) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, host_logits) == cudaSuccess)
      pinned = pa.type == cudaMemoryTypeHost;
    else
      (void)cudaGetLastError();  // not a CUDA pointer: leave no error for the next launch check
  }
  if (host_logits)
    GB_CUDA(cudaMemcpyAsync(pinned ? host_logits : m->h_logits, src, sizeof(float) * (size_t)m->c.vocab,
                            cudaMemcpyDeviceToHost, m->st),
            "model: logits");
  if ((rc = check_err(m))) return rc;
  if (host_logits && !pinned) memcpy(host_logits, m->h_logits, sizeof(float) * (size_t)m->c.vocab);
  return GB_OK;
}

int gb_model_next(gb_model *m, int32_t token, int pos, int32_t *next) {
  gb_clear_error();
  if (!m || !next) return gb_fail(GB_ERR_INVALID, "model: null argument");
  int rc = set_token_pos(m, token, pos);
  if (rc || (rc = run_step(m))) return rc;
  GB_CUDA(cudaMemcpyAsync(m->h_stage + 2, m->token, sizeof(int32_t), cudaMemcpyDeviceToHost, m->st), "model: token");
  if ((rc = check_err(m))) return rc;
  *next = m->h_stage[2];
  return GB_OK;
}

int gb_model_generate(gb_model *m, int32_t token, int pos, int n, int32_t *out_tokens) {
  gb_clear_error();
  if (!m || n < 0 || (n > 0 && !out_tokens)) return gb_fail(GB_ERR_INVALID, "model: bad generate arguments");
  if (pos + n > m->c.max_len)
    return gb_fail(GB_ERR_INVALID, "model: %d steps from position %d exceed the %d-token cache", n, pos, m->c.max_len);
  int rc = set_token_pos(m, token, pos);
  if (rc) return rc;
  for (int i = 0; i < n; i++)
    if ((rc = run_step(m))) return rc;
  if (n > 0)
    GB_CUDA(cudaMemcpyAsync(out_tokens, m->gen + pos, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToHost, m->st),
            "model: tokens");
  return check_err(m);
}


int gb_model_prefill(gb_model *m, const int32_t *tokens, int n, int pos0, float *host_logits) {
  gb_clear_error();
  if (!m || !tokens || n <= 0) return gb_fail(GB_ERR_INVALID, "model: bad prefill arguments");
  if (pos0 < 0 || pos0 + n > m->c.max_len)
    return gb_fail(GB_ERR_INVALID, "model: %d tokens from position %d exceed the %d-token cache", n, pos0,
                   m->c.max_len);
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= m->c.vocab)
      return gb_fail(GB_ERR_INVALID, "model: token %d outside the vocabulary", tokens[i]);
  int rc;
  if (n > 1 && (rc = prefill_workspace(m))) return rc;
  for (int c0 = 0; c0 < n - 1; c0 += kPrefillChunk) {
    const int T = std::min(kPrefillChunk, n - 1 - c0);
    GB_CUDA(cudaMemcpyAsync(m->pf_tokens, tokens + c0, sizeof(int32_t) * (size_t)T, cudaMemcpyHostToDevice, m->st),
            "model: prefill tokens");
    if ((rc = prefill_chunk(m, T, pos0 + c0))) return rc;
    GB_CUDA(cudaStreamSynchronize(m->st), "model: prefill");  // the next chunk's tokens reuse the buffer
  }
  // the last token through the decode step: its logits, and its own K/V
  return gb_model_forward(m, tokens[n - 1], pos0 + n - 1, host_logits);
}

int gb_model_cache_f16_weights(gb_model *m, size_t *bytes) {
  gb_clear_error();
  if (!m) return gb_fail(GB_ERR_INVALID, "model: null model");
  // every matrix with the GEMM arguments it is used with (the gate/up pairs
  // as one half's rows and tiles)
  std::vector<std::pair<Tiled *, GbTcGemm>> mats;
  for (auto &L : m->layers) {
    mats.emplace_back(&L.qkv, tc_args(L.qkv, GB_EPI_PLAIN, 0, m->pf_map_dim, m));
    mats.emplace_back(&L.wo, tc_args(L.wo, GB_EPI_RESID, 0, m->pf_map_q, m));
    GbTcGemm g = tc_args(L.gu, GB_EPI_SWIGLU, 0, m->pf_map_dim, m);
    g.rows = m->ffn_local;
    g.ntiles = L.gu.ntiles / 2;
    mats.emplace_back(&L.gu, g);
    mats.emplace_back(&L.down, tc_args(L.down, GB_EPI_RESID, 0, m->pf_map_ffn, m));
  }
  mats.emplace_back(&m->head, tc_args(m->head, GB_EPI_PLAIN, 0, m->pf_map_dim, m));
  size_t need = 0;
  for (auto &e : mats)
    if (!e.first->w16) need += gb_tc_f16_rows(e.second) * (size_t)e.second.nsb * 256 * sizeof(__half);
  if (bytes) *bytes = need;
  if (!need) return GB_OK;
  size_t free_b = 0, total_b = 0;
  GB_CUDA(cudaSetDevice(m->o.device), "model: binary16 weights");
  GB_CUDA(cudaMemGetInfo(&free_b, &total_b), "model: binary16 weights");
  if (need + ((size_t)1 << 30) > free_b)  // keep 1 GiB for the caller's workspaces
    return gb_fail(GB_ERR_UNSUPPORTED, "model: binary16 weights need %.2f GB, %.2f GB free", need / 1e9, free_b / 1e9);
  for (auto &e : mats) {
    Tiled &t = *e.first;
    if (t.w16) continue;
    __half *w16 = nullptr;
    int rc = dalloc(m, &w16, gb_tc_f16_rows(e.second) * (size_t)e.second.nsb * 256, "model: binary16 weights");
    if (!rc) rc = gb_tc_f16_weights_launch(e.second, w16, &t.map16, m->st);
    if (rc) return rc;
    t.w16 = w16;
  }
  GB_CUDA(cudaStreamSynchronize(m->st), "model: binary16 weights");
  return GB_OK;
}

int gb_linear_matmul_f16(gb_linear *l, void *stream, const uint16_t *x, int T, float *y) {
  gb_clear_error();
  if (!l || !x || !y || T < 0) return gb_fail(GB_ERR_INVALID, "model: linear: bad matmul arguments");
  if ((uintptr_t)x % 16 || (uintptr_t)y % 16) return gb_fail(GB_ERR_INVALID, "model: linear: x and y must be 16-byte aligned");
  if (T == 0) return GB_OK;
  GbTcGemm g;
  g.w = l->t.w;
  g.type_a = g.type_b = l->t.type_a;
  g.rows = l->t.rows;
  g.ntiles = l->t.ntiles;
  g.nsb = l->t.nsb;
  g.epi = GB_EPI_PLAIN;
  g.T = T;
  g.y = y;
  g.ldy = l->t.rows;
  int rc = gb_tmap_f16_rows(x, T, l->t.cols, &g.tmap_a);
  if (!rc) rc = gb_tmap_f16_rows(x, T, l->t.cols, &g.tmap_a16, 16);
  if (rc) return rc;
  g.a16 = true;
  if (l->t.w16) {
    g.w16 = l->t.w16;
    g.tmap_b = l->t.map16;
  }
  const GbTcPlan plan = gb_tc_gemm_plan(g, 148);
  if (plan.part_floats > l->mm_part_floats) {
    // the first call (or a larger T) grows the split-K scratch; the device
    // is synchronized first, as a previous launch may still read the old one
    GB_CUDA(cudaDeviceSynchronize(), "model: linear: matmul scratch");
    if (l->mm_part) cudaFree(l->mm_part);
    l->mm_part = nullptr;
    l->mm_part_floats = 0;
    GB_CUDA(cudaMalloc(&l->mm_part, plan.part_floats * sizeof(float)), "model: linear: matmul scratch");
    l->mm_part_floats = plan.part_floats;
  }
  g.part = l->mm_part;
  g.part_floats = l->mm_part_floats;
  return gb_tc_gemm_launch(g, (cudaStream_t)stream);
}

int gb_linear_cache_f16_weights(gb_linear *l, size_t *bytes) {
  gb_clear_error();
  if (!l) return gb_fail(GB_ERR_INVALID, "model: linear: null linear");
  GbTcGemm g;
  g.w = l->t.w;
  g.type_a = g.type_b = l->t.type_a;
  g.rows = l->t.rows;
  g.ntiles = l->t.ntiles;
  g.nsb = l->t.nsb;
  g.epi = GB_EPI_PLAIN;
  const size_t n = gb_tc_f16_rows(g) * (size_t)g.nsb * 256;
  if (bytes) *bytes = n * sizeof(__half);
  if (l->t.w16) return GB_OK;
  GB_CUDA(cudaSetDevice(l->device), "model: linear: binary16 weights");
  __half *w16 = nullptr;
  GB_CUDA(cudaMalloc(&w16, n * sizeof(__half)), "model: linear: binary16 weights");
  int rc = gb_tc_f16_weights_launch(g, w16, &l->t.map16, nullptr);
  if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = gb_fail(GB_ERR_CUDA, "model: linear: binary16 weights");
  if (rc) {
    cudaFree(w16);
    return rc;
  }
  l->t.w16 = w16;
  return GB_OK;
}

}  // extern "C"

// ---- continuous batching: a decode step for many sequences at once ---------
// Every active sequence owns pages of a paged KV pool (per layer
// [n_pages][n_kv][page_size][head_dim] binary16); a step takes one token per
// listed sequence and runs them as the rows of one batched pass (the
// prefill kernels: tensor-core GEMMs over binary16 activations, RoPE/KV
// append through the page tables, the paged attention), then the output
// RMSNorm, the lm_head GEMM and a first-maximum argmax per row.
struct gb_engine {
  gb_model *m = nullptr;
  int page_size = 0, n_pages = 0, max_batch = 0, max_pages = 0, max_pos = 0;
  std::vector<uint16_t *> kpool, vpool;
  std::vector<int> free_pages;
  struct Seq {
    bool live = false;
    int len = 0;
    std::vector<int> pages;
  };
  std::vector<Seq> seqs;
  float *logits = nullptr, *part = nullptr;
  size_t part_floats = 0;
  unsigned *counter = nullptr;
  int32_t *d_in = nullptr;   // tokens [B] | pos [B] | lens [B] | table [B][max_pages] | groups [B + 1]
  int32_t *h_in = nullptr;   // pinned copy of d_in
  int32_t *d_next = nullptr;
  std::vector<void *> allocs;
  // one CUDA graph of the step per (rows, attention splits, row groups) met so far
  std::map<std::tuple<int, int, int>, cudaGraphExec_t> graphs;
  std::vector<int> row_off;  // per sequence: rows of the current step so far
};

namespace {

constexpr size_t kEngineGraphs = 64;  // graphs kept before the cache is emptied

void drop_graphs(gb_engine *e) {
  for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
  e->graphs.clear();
}

void free_engine(gb_engine *e) {
  if (!e) return;
  if (e->m && e->m->st) cudaStreamSynchronize(e->m->st);
  drop_graphs(e);
  for (void *p : e->allocs) cudaFree(p);
  if (e->h_in) cudaFreeHost(e->h_in);
  delete e;
}

template <class T>
int ealloc(gb_engine *e, T **p, size_t n, const char *what) {
  void *q = nullptr;
  GB_CUDA(cudaMalloc(&q, std::max<size_t>(n * sizeof(T), 16)), what);
  GB_CUDA(cudaMemsetAsync(q, 0, std::max<size_t>(n * sizeof(T), 16), e->m->st), what);
  e->allocs.push_back(q);
  *p = (T *)q;
  return GB_OK;
}

// Paged attention splits for n rows whose longest sequence has max_len
// positions: about two CTAs per SM, within the scratch, and no more than
// give each split's warps one 32-position chunk each.
int engine_splits(const gb_engine *e, int n, int ngroups, int max_len) {
  const gb_model *m = e->m;
  const int hd = m->c.head_dim, nkv = m->kv_local / hd, G = m->c.heads / m->c.kv_heads;
  long long S = (2LL * m->sms + (long long)nkv * ngroups - 1) / ((long long)nkv * ngroups);
  S = std::min<long long>(S, std::max(1, (max_len + 32 * 8 - 1) / (32 * 8)));
  S = std::min<long long>(S, 32);
  S = std::min<long long>(S, (long long)(e->part_floats / gb_paged_part_floats(n, nkv, 1, G, hd)));
  return (int)std::max<long long>(S, 1);
}

int engine_forward(gb_engine *e, int n, int S, int ngroups) {
  gb_model *m = e->m;
  const gb_config &c = m->c;
  cudaStream_t st = m->st;
  const int hd = c.head_dim, qkv = m->q_local + 2 * m->kv_local, nkv = m->kv_local / hd;
  const int32_t *tok = e->d_in, *pos = e->d_in + e->max_batch, *lens = e->d_in + 2 * e->max_batch,
                *table = e->d_in + 3 * e->max_batch;
  const int32_t *groups = ngroups < n ? table + (size_t)e->max_batch * e->max_pages : nullptr;
  int rc = gb_embed_rows_launch(m->embd_type, m->embd.w, m->embd_nsb, c.dim, tok, n, c.vocab, m->pf_x, nullptr, 0,
                                c.max_len, m->err, st);
  if (rc) return rc;
  for (int l = 0; l < c.layers; l++) {
    gb_model::Layer &L = m->layers[(size_t)l];
    if ((rc = gb_rmsnorm_rows_f16_launch(m->pf_x, L.attn_norm, n, c.dim, c.eps, m->pf_a16, st))) return rc;
    GbTcGemm g = tc_args(L.qkv, GB_EPI_PLAIN, n, m->pf_map_dim, m);
    g.y = m->pf_qkv;
    g.ldy = qkv;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
    if ((rc = gb_rope_kv_paged_launch(m->pf_qkv, n, m->q_local, m->kv_local, hd, m->rope_cs, pos, table, e->max_pages,
                                      e->page_size, e->n_pages, c.max_len, m->pf_q, e->kpool[(size_t)l],
                                      e->vpool[(size_t)l], m->err, st)))
      return rc;
    if ((rc = gb_attn_paged_launch(m->pf_q, e->kpool[(size_t)l], e->vpool[(size_t)l], 1, table, lens, n, e->max_pages,
                                   e->n_pages, e->page_size, m->q_local / hd, nkv, hd, 1.f / sqrtf((float)hd),
                                   nullptr, m->pf_a16, e->part, e->counter, (int)S, m->err, st, groups, ngroups)))
      return rc;
    g = tc_args(L.wo, GB_EPI_RESID, n, m->pf_map_q, m);
    g.y = m->pf_x;
    g.ldy = c.dim;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
    if ((rc = gb_rmsnorm_rows_f16_launch(m->pf_x, L.ffn_norm, n, c.dim, c.eps, m->pf_a16, st))) return rc;
    g = tc_args(L.gu, GB_EPI_SWIGLU, n, m->pf_map_dim, m);
    g.rows = m->ffn_local;
    g.ntiles = L.gu.ntiles / 2;
    g.act = m->pf_act16;
    g.ld_act = m->ffn_local;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
    g = tc_args(L.down, GB_EPI_RESID, n, m->pf_map_ffn, m);
    g.y = m->pf_x;
    g.ldy = c.dim;
    if ((rc = gb_tc_gemm_launch(g, st))) return rc;
  }
  if ((rc = gb_rmsnorm_rows_f16_launch(m->pf_x, m->out_norm, n, c.dim, c.eps, m->pf_a16, st))) return rc;
  GbTcGemm g = tc_args(m->head, GB_EPI_PLAIN, n, m->pf_map_dim, m);
  g.y = e->logits;
  g.ldy = c.vocab;
  if ((rc = gb_tc_gemm_launch(g, st))) return rc;
  return gb_argmax_rows_launch(e->logits, n, c.vocab, e->d_next, st);
}

}  // namespace

extern "C" {

int gb_engine_create(gb_model *m, int page_size, int n_pages, int max_batch, gb_engine **out) {
  gb_clear_error();
  if (!m || !out || page_size <= 0 || n_pages <= 0 || max_batch <= 0)
    return gb_fail(GB_ERR_INVALID, "engine: bad arguments");
  if (m->c.tp_world > 1) return gb_fail(GB_ERR_UNSUPPORTED, "engine: continuous batching under tensor parallelism");
  if (max_batch > kPrefillChunk)
    return gb_fail(GB_ERR_UNSUPPORTED, "engine: at most %d sequences a step", kPrefillChunk);
  if (m->c.head_dim % 32 || m->c.head_dim > 128 || m->c.heads / m->c.kv_heads > 8)
    return gb_fail(GB_ERR_UNSUPPORTED, "engine: head_dim %d, %d query heads per KV head", m->c.head_dim,
                   m->c.heads / m->c.kv_heads);
  int rc = prefill_workspace(m);
  if (rc) return rc;
  std::unique_ptr<gb_engine, void (*)(gb_engine *)> e(new gb_engine, free_engine);
  e->m = m;
  e->page_size = page_size;
  e->n_pages = n_pages;
  e->max_batch = max_batch;
  e->max_pos = m->c.max_len;  // the RoPE table's positions
  e->max_pages = (e->max_pos + page_size - 1) / page_size;
  const gb_config &c = m->c;
  const int hd = c.head_dim, nkv = m->kv_local / hd, G = c.heads / c.kv_heads;
  const size_t pool = (size_t)n_pages * nkv * page_size * hd;
  e->kpool.resize((size_t)c.layers);
  e->vpool.resize((size_t)c.layers);
  for (int l = 0; l < c.layers; l++)
    if ((rc = ealloc(e.get(), &e->kpool[(size_t)l], pool, "engine: KV pool")) ||
        (rc = ealloc(e.get(), &e->vpool[(size_t)l], pool, "engine: KV pool")))
      return rc;
  e->part_floats = gb_paged_part_floats(max_batch, nkv, 4, G, hd);
  if ((rc = ealloc(e.get(), &e->logits, (size_t)max_batch * c.vocab, "engine: work")) ||
      (rc = ealloc(e.get(), &e->part, e->part_floats, "engine: work")) ||
      (rc = ealloc(e.get(), &e->counter, (size_t)max_batch * nkv, "engine: work")) ||
      (rc = ealloc(e.get(), &e->d_in, (size_t)max_batch * (4 + e->max_pages) + 1, "engine: work")) ||
      (rc = ealloc(e.get(), &e->d_next, (size_t)max_batch, "engine: work")))
    return rc;
  GB_CUDA(cudaMallocHost(&e->h_in, sizeof(int32_t) * ((size_t)max_batch * (4 + e->max_pages) + 1)), "engine: staging");
  for (int p = n_pages - 1; p >= 0; p--) e->free_pages.push_back(p);
  GB_CUDA(cudaStreamSynchronize(m->st), "engine: create");
  *out = e.release();
  return GB_OK;
}

int gb_engine_add(gb_engine *e, int *seq_id) {
  gb_clear_error();
  if (!e || !seq_id) return gb_fail(GB_ERR_INVALID, "engine: null argument");
  for (size_t i = 0; i < e->seqs.size(); i++)
    if (!e->seqs[i].live) {
      e->seqs[i] = gb_engine::Seq();
      e->seqs[i].live = true;
      *seq_id = (int)i;
      return GB_OK;
    }
  e->seqs.emplace_back();
  e->seqs.back().live = true;
  *seq_id = (int)e->seqs.size() - 1;
  return GB_OK;
}

int gb_engine_release(gb_engine *e, int seq_id) {
  gb_clear_error();
  if (!e || seq_id < 0 || seq_id >= (int)e->seqs.size() || !e->seqs[(size_t)seq_id].live)
    return gb_fail(GB_ERR_INVALID, "engine: no sequence %d", seq_id);
  gb_engine::Seq &q = e->seqs[(size_t)seq_id];
  for (int p : q.pages) e->free_pages.push_back(p);
  q = gb_engine::Seq();
  return GB_OK;
}

int gb_engine_seq_len(const gb_engine *e, int seq_id) {
  if (!e || seq_id < 0 || seq_id >= (int)e->seqs.size() || !e->seqs[(size_t)seq_id].live) return -1;
  return e->seqs[(size_t)seq_id].len;
}

int gb_engine_free_pages(const gb_engine *e) { return e ? (int)e->free_pages.size() : -1; }

int gb_engine_step(gb_engine *e, int n, const int32_t *seq_ids, const int32_t *tokens, float *host_logits,
                   int32_t *next) {
  gb_clear_error();
  if (!e || n <= 0 || !seq_ids || !tokens) return gb_fail(GB_ERR_INVALID, "engine: bad step arguments");
  if (n > e->max_batch) return gb_fail(GB_ERR_INVALID, "engine: %d rows, at most %d", n, e->max_batch);
  gb_model *m = e->m;
  // validate every row before touching any state. A sequence listed k times
  // feeds k tokens at its next k positions, in the order listed (a prompt
  // chunk); each row attends to its sequence's positions up to its own.
  std::vector<int> &off = e->row_off;
  off.assign(e->seqs.size(), 0);
  int need_pages = 0;
  for (int t = 0; t < n; t++) {
    const int id = seq_ids[t];
    if (id < 0 || id >= (int)e->seqs.size() || !e->seqs[(size_t)id].live)
      return gb_fail(GB_ERR_INVALID, "engine: no sequence %d", id);
    if (tokens[t] < 0 || tokens[t] >= m->c.vocab)
      return gb_fail(GB_ERR_INVALID, "model: token %d outside the vocabulary", tokens[t]);
    const gb_engine::Seq &q = e->seqs[(size_t)id];
    const int pos = q.len + off[(size_t)id]++;
    if (pos >= e->max_pos) return gb_fail(GB_ERR_INVALID, "engine: sequence %d is full (%d positions)", id, pos);
    if (pos % e->page_size == 0 && (int)q.pages.size() <= pos / e->page_size) need_pages++;
  }
  if (need_pages > (int)e->free_pages.size())
    return gb_fail(GB_ERR_UNSUPPORTED, "engine: out of KV pages (%d needed, %zu free)", need_pages,
                   e->free_pages.size());
  int32_t *h = e->h_in;
  const int B = e->max_batch;
  int max_len = 0;
  off.assign(e->seqs.size(), 0);
  for (int t = 0; t < n; t++) {
    gb_engine::Seq &q = e->seqs[(size_t)seq_ids[t]];
    const int pos = q.len + off[(size_t)seq_ids[t]]++;
    max_len = std::max(max_len, pos + 1);
    if ((int)q.pages.size() <= pos / e->page_size) {  // this position starts a page
      q.pages.push_back(e->free_pages.back());
      e->free_pages.pop_back();
    }
    h[t] = tokens[t];
    h[B + t] = pos;
    h[2 * B + t] = pos + 1;
  }
  // page tables after the step's allocations (a row attends only up to its
  // own position, so later pages of its sequence are harmless), and row
  // groups: consecutive rows of one sequence, up to the attention's group size
  const int R = gb_attn_paged_group_rows(m->c.heads / m->c.kv_heads);
  int32_t *grp = h + 3 * B + (size_t)B * e->max_pages;
  int ngroups = 0;
  for (int t = 0; t < n; t++) {
    const gb_engine::Seq &q = e->seqs[(size_t)seq_ids[t]];
    int32_t *row = h + 3 * B + (size_t)t * e->max_pages;
    for (int i = 0; i < e->max_pages; i++) row[i] = i < (int)q.pages.size() ? q.pages[(size_t)i] : -1;
    if (t == 0 || seq_ids[t] != seq_ids[t - 1] || t - grp[ngroups - 1] >= R) grp[ngroups++] = t;
  }
  grp[ngroups] = n;
  GB_CUDA(cudaMemcpyAsync(e->d_in, h, sizeof(int32_t) * ((size_t)B * (4 + e->max_pages) + 1), cudaMemcpyHostToDevice,
                          m->st),
          "engine: step inputs");
  // the step's kernels: replayed from the graph of (n, S, groups), captured on first use
  const int S = engine_splits(e, n, ngroups, max_len);
  int rc = GB_OK;
  if (m->o.use_graph) {
    auto it = e->graphs.find(std::make_tuple(n, S, ngroups));
    if (it == e->graphs.end()) {
      if (e->graphs.size() >= kEngineGraphs) drop_graphs(e);
      cudaGraph_t g = nullptr;
      cudaGraphExec_t x = nullptr;
      GB_CUDA(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal), "engine: graph capture");
      rc = engine_forward(e, n, S, ngroups);
      const cudaError_t ce = cudaStreamEndCapture(m->st, &g);
      if (!rc && ce != cudaSuccess) rc = gb_cuda_fail(ce, "engine: graph capture");
      if (!rc && cudaGraphInstantiate(&x, g, 0) != cudaSuccess) rc = gb_fail(GB_ERR_CUDA, "engine: graph instantiate");
      if (g) cudaGraphDestroy(g);
      if (rc) return rc;
      it = e->graphs.emplace(std::make_tuple(n, S, ngroups), x).first;
    }
    rc = cudaGraphLaunch(it->second, m->st) == cudaSuccess ? GB_OK : gb_fail(GB_ERR_CUDA, "engine: graph launch");
  } else {
    rc = engine_forward(e, n, S, ngroups);
  }
  if (!rc && host_logits)
    rc = cudaMemcpyAsync(host_logits, e->logits, sizeof(float) * (size_t)n * m->c.vocab, cudaMemcpyDeviceToHost,
                         m->st) == cudaSuccess
             ? GB_OK
             : gb_fail(GB_ERR_CUDA, "engine: logits");
  if (!rc && next)
    rc = cudaMemcpyAsync(next, e->d_next, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToHost, m->st) == cudaSuccess
             ? GB_OK
             : gb_fail(GB_ERR_CUDA, "engine: tokens");
  if (!rc) rc = check_err(m);
  if (rc) return rc;
  for (int t = 0; t < n; t++) e->seqs[(size_t)seq_ids[t]].len++;
  return GB_OK;
}

int gb_engine_free(gb_engine *e) {
  gb_clear_error();
  free_engine(e);
  return GB_OK;
}

int gb_model_set_sampler(gb_model *m, const gb_sample_params *p) {
  gb_clear_error();
  if (!m) return gb_fail(GB_ERR_INVALID, "model: null model");
  if (!p) {
    m->sampling = false;
    return GB_OK;
  }
  if (m->c.tp_world > 1) return gb_fail(GB_ERR_UNSUPPORTED, "model: sampling under tensor parallelism");
  if (m->c.vocab > kSampleMaxVocab) return gb_fail(GB_ERR_UNSUPPORTED, "model: vocabulary too large to sample");
  if (p->top_p != p->top_p || p->temperature != p->temperature || p->repeat_penalty != p->repeat_penalty)
    return gb_fail(GB_ERR_INVALID, "model: NaN sampler parameter");
  // the graph reads the parameters from device memory: copy, then wait, so
  // the host struct may go away
  GB_CUDA(cudaMemcpyAsync(m->sample_p, p, sizeof *p, cudaMemcpyHostToDevice, m->st), "model: sampler");
  GB_CUDA(cudaStreamSynchronize(m->st), "model: sampler");
  if (m->o.use_graph && !m->graph_sample) {
    int rc = capture(m, true);
    if (rc) return rc;
  }
  m->sampling = true;
  return GB_OK;
}

int gb_model_start(gb_model *m, int32_t token, int pos) {
  gb_clear_error();
  if (!m) return gb_fail(GB_ERR_INVALID, "model: null model");
  return set_token_pos(m, token, pos);
}

int gb_model_decode_async(gb_model *m, int n) {
  gb_clear_error();
  if (!m || n < 0) return gb_fail(GB_ERR_INVALID, "model: bad decode arguments");
  for (int i = 0; i < n; i++) {
    int rc = run_step(m);
    if (rc) return rc;
  }
  return GB_OK;
}

int gb_model_read_tokens(gb_model *m, int pos0, int n, int32_t *out_tokens) {
  gb_clear_error();
  if (!m || pos0 < 0 || n < 0 || pos0 + n > m->c.max_len || (n > 0 && !out_tokens))
    return gb_fail(GB_ERR_INVALID, "model: bad token range");
  if (n > 0)
    GB_CUDA(cudaMemcpyAsync(out_tokens, m->gen + pos0, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToHost, m->st),
            "model: tokens");
  return check_err(m);
}

int gb_model_fill_kv_normal(gb_model *m, uint64_t seed, int n_pos) {
  gb_clear_error();
  if (!m || n_pos < 0 || n_pos > m->c.max_len) return gb_fail(GB_ERR_INVALID, "model: bad KV fill");
  const gb_config &c = m->c;
  const int hd = c.head_dim, kv_dim = c.kv_heads * hd, kvl = m->kv_local, h0 = c.tp_rank * kvl;
  const size_t esz = c.kv_f16 ? 2 : 4, elems = (size_t)kvl * c.max_len;
  std::vector<float> k((size_t)n_pos * kv_dim), v((size_t)n_pos * kv_dim);
  std::vector<uint8_t> kd(elems * esz, 0), vd(elems * esz, 0);
  const int V = c.kv_f16 ? 8 : 4;
  for (int l = 0; l < c.layers; l++) {
    int rc = gb_synth_kv_normal(seed, l, 0, n_pos, kv_dim, c.kv_f16, k.data(), v.data());
    if (rc) return rc;
    for (int t = 0; t < n_pos; t++)
      for (int j = 0; j < kvl; j++) {
        int h = j / hd, d = j % hd;
        float kx = k[(size_t)t * kv_dim + h0 + j], vx = v[(size_t)t * kv_dim + h0 + j];
        size_t ki = (((size_t)h * (hd / V) + d / V) * c.max_len + t) * V + d % V;
        size_t vi = c.kv_f16 ? ki : ((size_t)h * c.max_len + t) * hd + d;
        if (c.kv_f16) {
          ((uint16_t *)kd.data())[ki] = host_f16(kx);
          ((uint16_t *)vd.data())[vi] = host_f16(vx);
        } else {
          ((float *)kd.data())[ki] = kx;
          ((float *)vd.data())[vi] = vx;
        }
      }
    GB_CUDA(cudaMemcpyAsync(m->layers[(size_t)l].kc, kd.data(), kd.size(), cudaMemcpyHostToDevice, m->st),
            "model: KV fill");
    GB_CUDA(cudaMemcpyAsync(m->layers[(size_t)l].vc, vd.data(), vd.size(), cudaMemcpyHostToDevice, m->st),
            "model: KV fill");
    GB_CUDA(cudaStreamSynchronize(m->st), "model: KV fill");  // kd, vd are reused per layer
  }
  return GB_OK;
}

int gb_model_read_kv(gb_model *m, int layer, int pos0, int n, float *k_out, float *v_out) {
  gb_clear_error();
  if (!m || layer < 0 || layer >= m->c.layers || pos0 < 0 || n < 0 || pos0 + n > m->c.max_len)
    return gb_fail(GB_ERR_INVALID, "model: bad KV read");
  const gb_config &c = m->c;
  const int hd = c.head_dim, kvl = m->kv_local, V = c.kv_f16 ? 8 : 4;
  const size_t esz = c.kv_f16 ? 2 : 4, elems = (size_t)kvl * c.max_len;
  std::vector<uint8_t> kd(elems * esz), vd(elems * esz);
  GB_CUDA(cudaMemcpyAsync(kd.data(), m->layers[(size_t)layer].kc, kd.size(), cudaMemcpyDeviceToHost, m->st),
          "model: KV read");
  GB_CUDA(cudaMemcpyAsync(vd.data(), m->layers[(size_t)layer].vc, vd.size(), cudaMemcpyDeviceToHost, m->st),
          "model: KV read");
  GB_CUDA(cudaStreamSynchronize(m->st), "model: KV read");
  for (int t = 0; t < n; t++)
    for (int j = 0; j < kvl; j++) {
      int h = j / hd, d = j % hd, p = pos0 + t;
      size_t ki = (((size_t)h * (hd / V) + d / V) * c.max_len + p) * V + d % V;
      size_t vi = c.kv_f16 ? ki : ((size_t)h * c.max_len + p) * hd + d;
      k_out[(size_t)t * kvl + j] = c.kv_f16 ? host_half(((uint16_t *)kd.data())[ki]) : ((float *)kd.data())[ki];
      v_out[(size_t)t * kvl + j] = c.kv_f16 ? host_half(((uint16_t *)vd.data())[vi]) : ((float *)vd.data())[vi];
    }
  return GB_OK;
}

void *gb_model_stream(gb_model *m) { return m ? (void *)m->st : nullptr; }

int gb_model_profile_step(gb_model *m, int32_t token, int pos, float *ms_out, int *launches) {
  gb_clear_error();
  if (!m || !ms_out) return gb_fail(GB_ERR_INVALID, "model: null argument");
  std::unique_ptr<Hook> h(new Hook());
  for (int i = 0; i < 1024; i++) GB_CUDA(cudaEventCreate(&h->ev[i]), "model: profile events");
  int rc = set_token_pos(m, token, pos);
  if (!rc) rc = enqueue_step(m, m->st, h.get());
  if (!rc) rc = check_err(m);
  for (int c = 0; c < K_CLASSES; c++) {
    ms_out[c] = 0.f;
    if (launches) launches[c] = 0;
  }
  if (!rc) {
    for (int i = 1; i < h->n; i++) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, h->ev[i - 1], h->ev[i]);
      int c = h->cls[i];
      if (c >= 0 && c < K_CLASSES) {
        ms_out[c] += ms;
        if (launches) launches[c]++;
      }
    }
  }
  for (int i = 0; i < 1024; i++) cudaEventDestroy(h->ev[i]);
  return rc;
}

int gb_model_step_bytes(const gb_model *m, int kv_len, double *bytes_per_token, double *gateup_bytes) {
  gb_clear_error();
  if (!m) return gb_fail(GB_ERR_INVALID, "model: null model");
  const gb_config &c = m->c;
  double w = 0;
  for (auto &L : m->layers) w += (double)L.qkv.bytes + L.wo.bytes + L.gu.bytes + L.down.bytes;
  // tiled bytes include row padding only when rows are not multiples of 32
  w += (double)gb_row_bytes(m->head.type_a, c.dim) * m->vocab_local;
  double norms = 4.0 * c.dim * (2.0 * c.layers + 1);
  double esz = c.kv_f16 ? 2.0 : 4.0;
  double kv = (double)c.layers * (double)kv_len * 2.0 * m->kv_local * esz + (double)c.layers * 2.0 * m->kv_local * esz;
  double emb = (double)gb_row_bytes(m->embd_type, c.dim);
  if (bytes_per_token) *bytes_per_token = w + norms + kv + emb;
  if (gateup_bytes) *gateup_bytes = m->layers.empty() ? 0 : (double)m->layers[0].gu.bytes;
  return GB_OK;
}

int gb_model_launches_per_step(const gb_model *m) { return m ? m->launches : 0; }

int gb_model_close(gb_model *m) {
  gb_clear_error();
  if (m) {
    cudaStreamSynchronize(m->st);
    free_model(m);
  }
  return GB_OK;
}

int gb_tp_unique_id(uint8_t out[128]) {
  gb_clear_error();
  if (!nccl() || !nccl()->getUniqueId) return gb_fail(GB_ERR_NCCL, "tp: libnccl.so.2 not found");
  ncclUniqueId id;
  GB_NCCL(nccl()->getUniqueId(&id), "tp: unique id");
  memcpy(out, &id, 128);
  return GB_OK;
}

// ---- model.Linear ------------------------------------------------------------

static void free_linear(gb_linear *l) {
  if (!l) return;
  if (l->t.w) cudaFree(l->t.w);
  if (l->t.w16) cudaFree(l->t.w16);
  if (l->part) cudaFree(l->part);
  if (l->tile_counter) cudaFree(l->tile_counter);
  if (l->mm_part) cudaFree(l->mm_part);
  delete l;
}

int gb_linear_upload(int device, int typ, const void *host_bytes, size_t nbytes, int rows, int cols,
                     gb_linear **out) {
  gb_clear_error();
  if (!out || !host_bytes || rows <= 0 || cols <= 0) return gb_fail(GB_ERR_INVALID, "model: linear: bad arguments");
  if (!gb_tiled_type(typ)) return gb_fail(GB_ERR_UNSUPPORTED, "model: linear: no kernel for %s weights", tname(typ));
  if (cols % 256) return gb_fail(GB_ERR_UNSUPPORTED, "model: linear: %d columns is not a multiple of 256", cols);
  if (nbytes != (size_t)gb_row_bytes(typ, cols) * rows)
    return gb_fail(GB_ERR_INVALID, "model: linear: %zu bytes, want %lld", nbytes, (long long)gb_row_bytes(typ, cols) * rows);
  GB_CUDA(cudaSetDevice(device), "model: linear");
  gb_linear *l = new gb_linear();
  l->device = device;
  Tiled &t = l->t;
  t.type_a = t.type_b = typ;
  t.rows = rows;
  t.cols = cols;
  t.ntiles = (rows + 31) / 32;
  t.nsb = cols / 256;
  t.bytes = gb_tiled_bytes(typ, rows, cols);
  uint8_t *raw = nullptr;
  cudaError_t e = cudaMalloc(&t.w, t.bytes);
  if (e == cudaSuccess) e = cudaMalloc(&raw, nbytes);
  if (e == cudaSuccess) e = cudaMemcpy(raw, host_bytes, nbytes, cudaMemcpyHostToDevice);
  int rc = e == cudaSuccess ? gb_repack_launch(typ, raw, rows, cols, t.w, 0) : gb_cuda_fail(e, "model: linear upload");
  if (!rc) {
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) rc = gb_cuda_fail(e, "model: linear repack");
  }
  if (raw) cudaFree(raw);
  GbGemvPlan plan = gb_gemv_plan(t.ntiles, t.nsb, GB_EPI_PLAIN, 148);
  if (!rc && cudaMalloc(&l->part, sizeof(float) * (size_t)gb_gemv_scratch_floats(t.ntiles, plan)) != cudaSuccess)
    rc = gb_fail(GB_ERR_CUDA, "model: linear scratch");
  if (!rc && cudaMalloc(&l->tile_counter, sizeof(unsigned) * (size_t)(t.ntiles + 64)) != cudaSuccess)
    rc = gb_fail(GB_ERR_CUDA, "model: linear scratch");
  // a plain cudaMemset returns before a device-memory memset is done, and the
  // caller's stream may be non-blocking: finish it before the first product
  if (!rc && (cudaMemset(l->tile_counter, 0, sizeof(unsigned) * (size_t)(t.ntiles + 64)) != cudaSuccess ||
              cudaDeviceSynchronize() != cudaSuccess))
    rc = gb_fail(GB_ERR_CUDA, "model: linear scratch");
  if (rc) {
    free_linear(l);  // keeps the error message of the failed step
    return rc;
  }
  *out = l;
  return GB_OK;
}

int gb_linear_matvec(gb_linear *l, void *stream, const float *x, float *y) {
  gb_clear_error();
  if (!l) return gb_fail(GB_ERR_INVALID, "model: linear: null handle");
  if ((uintptr_t)x % 16) return gb_fail(GB_ERR_INVALID, "model: linear: x must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  GbGemvArgs a;
  a.w = l->t.w;
  a.type_a = a.type_b = l->t.type_a;
  a.rows = l->t.rows;
  a.ntiles = l->t.ntiles;
  a.nsb = l->t.nsb;
  a.in_x = x;
  a.epi = GB_EPI_PLAIN;
  a.e.y = y;
  a.e.part = l->part;
  a.e.tile_counter = l->tile_counter;
  // programmatic dependent launch: the weight stream (constant since the
  // upload) starts while the stream's previous kernel finishes; x is read and
  // y written only after that kernel has completed
  return gb_gemv_launch(a, gb_gemv_plan(l->t.ntiles, l->t.nsb, GB_EPI_PLAIN, 148), st, true);
}

int gb_linear_info(const gb_linear *l, int *typ, int *rows, int *cols, size_t *weight_bytes) {
  gb_clear_error();
  if (!l) return gb_fail(GB_ERR_INVALID, "model: linear: null handle");
  if (typ) *typ = l->t.type_a;
  if (rows) *rows = l->t.rows;
  if (cols) *cols = l->t.cols;
  if (weight_bytes) *weight_bytes = (size_t)gb_row_bytes(l->t.type_a, l->t.cols) * l->t.rows;
  return GB_OK;
}

int gb_linear_free(gb_linear *l) {
  gb_clear_error();
  free_linear(l);
  return GB_OK;
}

}  // extern "C"
