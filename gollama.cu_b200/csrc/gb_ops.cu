// gb_ops.cu -- the per-kernel launch API of backend/gpu (backend/gpu/gpu.go:35-167)
// as sm_100a kernels behind a C ABI, plus the small kernels of the decode
// step (embedding lookup, residual+pack, argmax) and the library's error slot.
//
// Per-op kernels keep the reference's argument meaning (same buffers, same
// row/column conventions, in-place use allowed where the reference allows it)
// and follow backend/cpu/cpu.go's arithmetic where it is cheap to do so
// (float64 reductions for RMSNorm/Softmax, float64 exp/pow/sincos), so they
// meet the reference's tolerances with margin.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#if defined(__SSE2__) && !defined(__CUDA_ARCH__)
#include <emmintrin.h>
#endif

#include "gb_device.cuh"
#include "gb_internal.h"

// ---- error slot -----------------------------------------------------------
static thread_local std::string g_err;

int gb_fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
int gb_cuda_fail(cudaError_t e, const char *what) {
  (void)cudaGetLastError();  // a non-sticky error must not resurface at the next launch check
  return gb_fail(GB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
void gb_clear_error() { g_err.clear(); }

namespace {

// ---- per-op kernels ----------------------------------------------------------

// kernels.RMSNorm (kernels/rows.go:7), with cpu.RMSNorm's float64 sum.
__global__ void rmsnorm_kernel(const float *x, const float *w, float *out, int n, float eps) {
  const float *xr = x + (size_t)blockIdx.x * n;
  float *o = out + (size_t)blockIdx.x * n;
  __shared__ double red[32];
  double ss = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * (double)xr[i];
  for (int k = 16; k > 0; k >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, k);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    red[0] = t;
  }
  __syncthreads();
  float inv = (float)(1.0 / sqrt(red[0] / (double)n + (double)eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// kernels.Softmax (kernels/rows.go:23), with cpu.Softmax's float64 exp and sum.
__global__ void softmax_kernel(const float *x, float *out, int n) {
  const float *xr = x + (size_t)blockIdx.x * n;
  float *o = out + (size_t)blockIdx.x * n;
  __shared__ float fred[32];
  __shared__ double dred[32];
  __shared__ int nan_seen;
  if (threadIdx.x == 0) nan_seen = 0;
  __syncthreads();
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xr[i];
    if (isnan(v)) nan_seen = 1;  // Go's max propagates NaN
    m = fmaxf(m, v);
  }
  m = gb_warp_max(m);
  if ((threadIdx.x & 31) == 0) fred[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t = fmaxf(t, fred[i]);
    fred[0] = nan_seen ? NAN : t;
  }
  __syncthreads();
  m = fred[0];
  double s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float e = (float)exp((double)(xr[i] - m));
    o[i] = e;
    s += (double)e;
  }
  for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
  if ((threadIdx.x & 31) == 0) dred[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += dred[i];
    dred[0] = t;
  }
  __syncthreads();
  float inv = (float)(1.0 / dred[0]);
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = o[i] * inv;
}

// kernels.SiluMul (kernels/rows.go:45).
__global__ void silu_mul_kernel(const float *g, const float *u, float *out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float gv = g[i];
    float e = (float)exp(-(double)gv);
    out[i] = gv / (1.f + e) * u[i];
  }
}

// kernels.Add (kernels/rows.go:54).
__global__ void add_kernel(const float *a, const float *b, float *out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = a[i] + b[i];
}

// kernels.RoPE (kernels/rows.go:67), angles and rotation in float64 as in
// cpu.RoPE (backend/cpu/cpu.go:69).
__global__ void rope_kernel(float *x, const int32_t *pos, const float *freq, int n_heads,
                            int head_dim, float base) {
  const int r = blockIdx.x, half = head_dim / 2;
  const double p = (double)pos[r];
  float *row = x + (size_t)r * n_heads * head_dim;
  for (int i = threadIdx.x; i < n_heads * half; i += blockDim.x) {
    int h = i / half, j = i % half;
    double theta = p * pow((double)base, -2.0 * (double)j / (double)head_dim);
    theta = theta / (double)freq[j];
    double s, c;
    sincos(theta, &s, &c);
    float *pr = row + h * head_dim + 2 * j;
    double x0 = pr[0], x1 = pr[1];
    pr[0] = (float)__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, s));
    pr[1] = (float)__dadd_rn(__dmul_rn(x0, s), __dmul_rn(x1, c));
  }
}

// kernels.MatVecF16 / MatVecF32 (kernels/matvec.go:10,30): one warp per row.
template <bool F16>
__global__ void matvec_dense_kernel(const void *w, const float *x, float *y, int rows, int cols) {
  int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int b = blockIdx.y, lane = threadIdx.x & 31;
  const float *xb = x + (size_t)b * cols;
  double acc = 0;
  for (int c = lane; c < cols; c += 32) {
    float wv = F16 ? gb_half_to_float(((const uint16_t *)w)[(size_t)r * cols + c])
                   : ((const float *)w)[(size_t)r * cols + c];
    acc += (double)wv * (double)xb[c];
  }
  for (int k = 16; k > 0; k >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, k);
  if (lane == 0) y[(size_t)b * rows + r] = (float)acc;
}

// kernels.MatVecQ4_0/Q4K/Q6K on raw ggml bytes (kernels/quantmv.go:18-136):
// one warp per (row, batch vector); each lane decodes whole blocks with the
// bit-exact decoder and accumulates in float64 like cpu.MatVecQ.
__global__ void matvec_q_raw_kernel(int typ, const uint8_t *w, const float *x, float *y, int rows,
                                    int cols) {
  int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int b = blockIdx.y, lane = threadIdx.x & 31;
  const int bs = gb_block_size(typ), ts = gb_type_size(typ), nb = cols / bs;
  const uint8_t *wr = w + (size_t)r * nb * ts;
  const float *xb = x + (size_t)b * cols;
  double acc = 0;
  for (int blk = lane; blk < nb; blk += 32) {
    const uint8_t *p = wr + (size_t)blk * ts;
    float part = 0.f;
    for (int e = 0; e < bs; e++) part = fmaf(gb_dequant_elem(typ, p, e), xb[blk * bs + e], part);
    acc += (double)part;
  }
  for (int k = 16; k > 0; k >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, k);
  if (lane == 0) y[(size_t)b * rows + r] = (float)acc;
}

// quant.Row on the device (quant/quant.go:135): bit-exact.
__global__ void dequant_rows_kernel(int typ, const uint8_t *w, int cols, int row0, int nrows,
                                    float *out) {
  const int bs = gb_block_size(typ), ts = gb_type_size(typ);
  const long long rb = (long long)(cols / bs) * ts;
  long long total = (long long)nrows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int r = (int)(i / cols), c = (int)(i % cols);
    const uint8_t *blk = w + (long long)(row0 + r) * rb + (long long)(c / bs) * ts;
    out[i] = gb_dequant_elem(typ, blk, c % bs);
  }
}

// Single-CTA argmax with model.Argmax's rule (model/model.go:376).
__global__ void argmax_kernel(const float *x, int n, int32_t *out) {
  __shared__ unsigned long long red[32];
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (isnan(v)) v = i == 0 ? INFINITY : -INFINITY;
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    unsigned long long k = ((unsigned long long)b << 32) | (0xFFFFFFFFull - (unsigned)i);
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t = red[i] > t ? red[i] : t;
    *out = (int32_t)(0xFFFFFFFFu - (uint32_t)(t & 0xFFFFFFFFull));
  }
}

// Wait (bounded by p.wait_limit polls, each sleeping ~100 ns; the default
// 2^22 is about half a second) until rank q's flag of peer slot `slot`
// carries this step's value (read over NVLink for another rank); false on
// timeout.
GB_DEV bool peer_wait(const GbPeer &p, int slot, int q) {
  const unsigned ep = *p.epoch + 1u;
  const unsigned *f = p.flags[q] + slot;
  for (unsigned i = 0; i < p.wait_limit; i++) {
    if (gb_ld_acquire_sys(f) == ep) return true;
    __nanosleep(64);
  }
  return false;
}

// x += sum over ranks of the partials in peer slot `slot` (rank order, so
// every rank computes the same x), with per-32 sums of squares.
__global__ void peer_resid_kernel(GbPeer p, int slot, float *x, int n, float *ssq, unsigned *err) {
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < p.world && !peer_wait(p, slot, threadIdx.x)) {
    ok = 0;
    if (err) atomicOr(err, GB_DEVERR_TIMEOUT);
  }
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x, lane = threadIdx.x & 31;
  if (c >= n) return;  // n is a multiple of 32: whole warps leave together
  float sum = 0.f;
  if (ok)
    for (int q = 0; q < p.world; q++) sum += __ldcv(p.bufs[q] + (size_t)slot * p.dim + c);
  const float xn = x[c] + sum;
  x[c] = xn;
  const float ss = gb_warp_sum(xn * xn);
  if (lane == 0) ssq[c / 32] = ss;
}

// The token from every rank's argmax key in peer slot `slot` (the largest
// key: larger value, then lower index, as model.Argmax).
// The exchange of the model's row-split GEMVs. Rank q's partial of element c
// is the 64-bit word t.w[q][slot*dim + c] = (step + 1) << 32 | float bits,
// stored by that rank's GEMV epilogue with no fence or flag. Each thread
// loads its element's word from every rank at once (one NVLink round trip
// once they have landed), polls again only words whose tag is still an older
// step (bounded: wait_limit polls each, ~100 ns apart), then adds the values
// in rank order, so every rank computes the same bits. A wait that runs out
// leaves x[c] as it was and sets GB_DEVERR_TIMEOUT.
constexpr int kTagBatch = 8;
__global__ void peer_resid_tagged_kernel(const __grid_constant__ GbTagTable t, int world, const unsigned *step,
                                         unsigned wait_limit, int slot, int dim, float *x, int n, float *ssq,
                                         unsigned *err) {
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x, lane = threadIdx.x & 31;
  if (c >= n) return;  // n is a multiple of 32: whole warps leave together
  const unsigned ep = __ldcg(step) + 1u;
  const size_t off = (size_t)slot * dim + c;
  float sum = 0.f;
  bool ok = true;
  for (int q0 = 0; q0 < world && ok; q0 += kTagBatch) {
    unsigned long long w[kTagBatch];
#pragma unroll
    for (int i = 0; i < kTagBatch; i++)
      if (q0 + i < world) w[i] = gb_ld_relaxed_sys_u64(t.w[q0 + i] + off);
#pragma unroll
    for (int i = 0; i < kTagBatch; i++) {
      if (q0 + i >= world || !ok) continue;
      for (unsigned k = 0; (unsigned)(w[i] >> 32) != ep; k++) {
        if (k >= wait_limit) {
          ok = false;
          break;
        }
        __nanosleep(64);
        w[i] = gb_ld_relaxed_sys_u64(t.w[q0 + i] + off);
      }
      sum += __uint_as_float((unsigned)(w[i] & 0xFFFFFFFFull));
    }
  }
  if (!ok && err) atomicOr(err, GB_DEVERR_TIMEOUT);
  const float xn = ok ? x[c] + sum : x[c];
  x[c] = xn;
  const float ss = gb_warp_sum(xn * xn);
  if (lane == 0) ssq[c / 32] = ss;
}

__global__ void peer_argmax_kernel(GbPeer p, int slot, int32_t *token, int32_t *hist, const int32_t *pos,
                                   int max_len, unsigned *err) {
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < p.world && !peer_wait(p, slot, threadIdx.x)) {
    ok = 0;
    if (err) atomicOr(err, GB_DEVERR_TIMEOUT);
  }
  __syncthreads();
  if (threadIdx.x != 0 || !ok) return;
  unsigned long long t = 0;
  for (int q = 0; q < p.world; q++) {
    const unsigned long long k = __ldcv((const unsigned long long *)(p.bufs[q] + (size_t)slot * p.dim));
    t = k > t ? k : t;
  }
  const int32_t tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(t & 0xFFFFFFFFull));
  *token = tok;
  if (hist) {
    const int ps = *pos;
    if (ps >= 0 && ps < max_len) hist[ps] = tok;
  }
}

__global__ void advance_pos_kernel(int32_t *pos, unsigned *epoch) {
  *pos += 1;
  if (epoch) *epoch += 1u;
}

// Embedding lookup (model/model.go:326 quant.Row on the host, moved on the
// device): row *token of the tiled token_embd, bit-exact, into x, with the
// per-32 sums of squares the first RMSNorm needs.
__global__ void embed_kernel(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *token,
                             int vocab, float *x, float *ssq, unsigned *err, int32_t *fed, const int32_t *pos,
                             int max_len) {
  __shared__ __align__(16) uint8_t blk[8][1024];  // one super-block of one row (F32: 1024 B)
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * (blockDim.x >> 5) + warp;
  if (g >= dim / 32) return;
  int tok = *token;
  if (fed && g == 0 && lane == 0) {
    // the token fed at this position (the sampler's repetition window)
    const int p = *pos;
    if (p >= 0 && p < max_len) fed[p] = tok;
  }
  if (tok < 0 || tok >= vocab) {
    if (g == 0 && lane == 0 && err) atomicOr(err, GB_DEVERR_TOKEN);
    tok = 0;
  }
  const int tile = tok / 32, tl = tok % 32, sb = g / 8;
  const int sbb = gb_tiled_sb_bytes(typ), raw = gb_sb_raw_bytes(typ);
  const uint8_t *base = tiled + ((size_t)tile * nsb + sb) * sbb;
  for (int b = lane; b < raw; b += 32) blk[warp][b] = base[gb_tiled_offset(typ, tl, b)];
  __syncwarp();
  int e = (g % 8) * 32 + lane;  // element within the super-block
  float v = typ == GB_T_Q4_0   ? gb_dequant_elem(typ, blk[warp] + 18 * (e / 32), e % 32)
            : typ == GB_T_Q8_0 ? gb_dequant_elem(typ, blk[warp] + 34 * (e / 32), e % 32)
                               : gb_dequant_elem(typ, blk[warp], e);
  x[g * 32 + lane] = v;
  float ss = gb_warp_sum(v * v);
  if (lane == 0) ssq[g] = ss;
}

// x += y with per-32 sums of squares: the residual epilogue when the
// projection's sum arrives from a collective.
__global__ void resid_kernel(float *x, const float *y, int n, float *ssq) {
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (g >= n / 32) return;
  int c = g * 32 + lane;
  float xn = x[c] + y[c];
  x[c] = xn;
  float ss = gb_warp_sum(xn * xn);
  if (lane == 0) ssq[g] = ss;
}

__global__ void fill_kernel(float *p, int n, float v) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute *attr,
                            bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

int blocks_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return b < 1 ? 1 : (int)b;
}

const char *type_name(int t) {
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
  return "unknown";
}

}  // namespace

// ---- internal launchers -----------------------------------------------------

int gb_embed_launch(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *token,
                    int vocab, float *x, float *ssq, unsigned *err, int32_t *fed, const int32_t *pos, int max_len,
                    cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  int groups = dim / 32;
  cudaLaunchConfig_t cfg = make_cfg(dim3((groups + 7) / 8), dim3(256), st, attr, pdl);
  GB_CUDA(cudaLaunchKernelEx(&cfg, embed_kernel, typ, tiled, nsb, dim, token, vocab, x, ssq, err, fed, pos,
                             max_len),
          "gpu: embed");
  return GB_OK;
}

int gb_add_launch(const float *a, const float *b, float *out, int n, cudaStream_t st) {
  add_kernel<<<blocks_for(n, 256), 256, 0, st>>>(a, b, out, n);
  GB_CUDA(cudaGetLastError(), "gpu: add");
  return GB_OK;
}

int gb_resid_launch(float *x, const float *y, int n, float *ssq, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  int groups = n / 32;
  cudaLaunchConfig_t cfg = make_cfg(dim3((groups + 7) / 8), dim3(256), st, attr, pdl);
  GB_CUDA(cudaLaunchKernelEx(&cfg, resid_kernel, x, y, n, ssq), "gpu: residual");
  return GB_OK;
}

int gb_peer_resid_launch(const GbPeer &p, int slot, float *x, int n, float *ssq, unsigned *err,
                         cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3((n + 255) / 256), dim3(256), st, attr, pdl);
  GB_CUDA(cudaLaunchKernelEx(&cfg, peer_resid_kernel, p, slot, x, n, ssq, err), "gpu: peer residual");
  return GB_OK;
}

int gb_peer_resid_tagged_launch(const GbTagTable &t, int world, const unsigned *step, unsigned wait_limit, int slot,
                                int dim, float *x, int n, float *ssq, unsigned *err, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3((n + 255) / 256), dim3(256), st, attr, pdl);
  GB_CUDA(cudaLaunchKernelEx(&cfg, peer_resid_tagged_kernel, t, world, step, wait_limit, slot, dim, x, n, ssq, err),
          "gpu: peer residual");
  return GB_OK;
}
int gb_peer_argmax_launch(const GbPeer &p, int slot, int32_t *token, int32_t *hist, const int32_t *pos,
                          int max_len, unsigned *err, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(32), st, attr, pdl);
  GB_CUDA(cudaLaunchKernelEx(&cfg, peer_argmax_kernel, p, slot, token, hist, pos, max_len, err),
          "gpu: peer argmax");
  return GB_OK;
}

int gb_advance_pos_launch(int32_t *pos, unsigned *epoch, cudaStream_t st) {
  advance_pos_kernel<<<1, 1, 0, st>>>(pos, epoch);
  GB_CUDA(cudaGetLastError(), "gpu: advance position");
  return GB_OK;
}

// ---- C ABI: backend/gpu ------------------------------------------------------

struct gb_kernels {
  int device = 0;
  unsigned *status = nullptr;  // device error word of calls given no status word of their own
  float *ws = nullptr;  // attention partials + counters
  size_t ws_floats = 0;
  unsigned *ws_counter = nullptr;
  int ws_nkv = 0;
  float *pws = nullptr;  // paged attention: split partials + counters
  size_t pws_floats = 0;
  unsigned *pws_counter = nullptr;
  size_t pws_counters = 0;
};

// The kernel names backend/gpu binds (backend/gpu/gpu.go:24); each has an
// entry point here.
static const char *const k_names[] = {"RMSNorm", "Softmax", "SiluMul", "Add", "RoPE", "MatVecF16",
                                      "MatVecF32", "MatVecQ4_0", "MatVecQ4K", "MatVecQ6K", "AttnDecode"};
static const int k_count = (int)(sizeof k_names / sizeof k_names[0]);

extern "C" {

const char *gb_last_error(void) { return g_err.c_str(); }
const char *gb_version(void) { return "gollama-b200 0.1 (sm_100a)"; }

int gb_gpu_load(int device, gb_kernels **out) {
  gb_clear_error();
  if (!out) return gb_fail(GB_ERR_INVALID, "gpu: load kernels: null handle");
  int n = 0;
  GB_CUDA(cudaGetDeviceCount(&n), "gpu: load kernels");
  if (device < 0 || device >= n) return gb_fail(GB_ERR_INVALID, "gpu: load kernels: no device %d", device);
  GB_CUDA(cudaSetDevice(device), "gpu: load kernels");
  cudaDeviceProp prop;
  GB_CUDA(cudaGetDeviceProperties(&prop, device), "gpu: load kernels");
  if (prop.major != 10)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: load kernels: device is sm_%d%d, the kernels are sm_100a",
                   prop.major, prop.minor);
  cudaFuncAttributes fa;
  GB_CUDA(cudaFuncGetAttributes(&fa, rmsnorm_kernel), "gpu: load kernels");
  gb_kernels *k = new gb_kernels();
  k->device = device;
  cudaError_t e = cudaMalloc(&k->status, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(k->status, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (k->status) cudaFree(k->status);
    delete k;
    return gb_cuda_fail(e, "gpu: load kernels");
  }
  *out = k;
  return GB_OK;
}

int gb_gpu_len(const gb_kernels *k) { return k && k_names[0] ? k_count : 0; }

int gb_gpu_close(gb_kernels *k) {
  gb_clear_error();
  if (!k) return GB_OK;
  if (k->ws) cudaFree(k->ws);
  if (k->ws_counter) cudaFree(k->ws_counter);
  if (k->pws) cudaFree(k->pws);
  if (k->pws_counter) cudaFree(k->pws_counter);
  if (k->status) cudaFree(k->status);
  delete k;
  return GB_OK;
}

#define GB_NEED(k)                                                        \
  do {                                                                    \
    if (!(k)) return gb_fail(GB_ERR_INVALID, "gpu: kernels not loaded"); \
  } while (0)

int gb_gpu_rmsnorm(gb_kernels *k, void *stream, const float *x, const float *w, float *out,
                   int rows, int n, float eps) {
  gb_clear_error();
  GB_NEED(k);
  if (rows <= 0 || n <= 0) return GB_OK;
  rmsnorm_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, w, out, n, eps);
  GB_CUDA(cudaGetLastError(), "gpu: RMSNorm");
  return GB_OK;
}

int gb_gpu_softmax(gb_kernels *k, void *stream, const float *x, float *out, int rows, int n) {
  gb_clear_error();
  GB_NEED(k);
  if (rows <= 0 || n <= 0) return GB_OK;
  softmax_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, out, n);
  GB_CUDA(cudaGetLastError(), "gpu: Softmax");
  return GB_OK;
}

int gb_gpu_silu_mul(gb_kernels *k, void *stream, const float *gate, const float *up, float *out, int n) {
  gb_clear_error();
  GB_NEED(k);
  if (n <= 0) return GB_OK;
  silu_mul_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(gate, up, out, n);
  GB_CUDA(cudaGetLastError(), "gpu: SiluMul");
  return GB_OK;
}

int gb_gpu_add(gb_kernels *k, void *stream, const float *a, const float *b, float *out, int n) {
  gb_clear_error();
  GB_NEED(k);
  if (n <= 0) return GB_OK;
  add_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(a, b, out, n);
  GB_CUDA(cudaGetLastError(), "gpu: Add");
  return GB_OK;
}

int gb_gpu_rope(gb_kernels *k, void *stream, float *x, const int32_t *pos, const float *freq,
                int rows, int n_heads, int head_dim, float base) {
  gb_clear_error();
  GB_NEED(k);
  if (head_dim % 2) return gb_fail(GB_ERR_INVALID, "gpu: RoPE: odd head_dim %d", head_dim);
  if (rows <= 0) return GB_OK;
  rope_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, pos, freq, n_heads, head_dim, base);
  GB_CUDA(cudaGetLastError(), "gpu: RoPE");
  return GB_OK;
}

int gb_gpu_attn_decode(gb_kernels *k, void *stream, const float *q, const float *kcache,
                       const float *vcache, float *out, int kv_len, int n_heads, int n_kv,
                       int head_dim, float scale) {
  gb_clear_error();
  GB_NEED(k);
  if (kv_len <= 0) return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: kv_len %d", kv_len);
  if (n_kv <= 0 || n_heads % n_kv)
    return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: %d heads is not a multiple of %d KV heads", n_heads, n_kv);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, k->device);
  int splits = (2 * sms + n_kv - 1) / n_kv;
  if (splits > 128) splits = 128;
  if (splits > kv_len) splits = kv_len;
  while ((kv_len + splits - 1) / splits > 2048) splits++;
  const int G = n_heads / n_kv;
  size_t need = gb_attn_part_floats(n_kv, splits, G, head_dim);
  if (need > k->ws_floats || n_kv > k->ws_nkv) {
    if (k->ws) cudaFree(k->ws);
    if (k->ws_counter) cudaFree(k->ws_counter);
    k->ws = nullptr;
    k->ws_counter = nullptr;
    k->ws_floats = 0;
    k->ws_nkv = 0;
    GB_CUDA(cudaMalloc(&k->ws, need * sizeof(float)), "gpu: AttnDecode: workspace");
    GB_CUDA(cudaMalloc(&k->ws_counter, sizeof(unsigned) * (size_t)n_kv), "gpu: AttnDecode: workspace");
    // on the call's stream: ordered before this launch whatever kind of stream it is
    GB_CUDA(cudaMemsetAsync(k->ws_counter, 0, sizeof(unsigned) * (size_t)n_kv, (cudaStream_t)stream),
            "gpu: AttnDecode: workspace");
    k->ws_floats = need;
    k->ws_nkv = n_kv;
  }
  GbAttnArgs a;
  a.q = q;
  a.k = kcache;
  a.v = vcache;
  a.kv_f16 = 0;
  const long long kv_dim = (long long)n_kv * head_dim;
  a.k_sh = head_dim;
  a.k_sd = 4;
  a.k_st = kv_dim;
  a.v_sh = head_dim;
  a.v_st = kv_dim;
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.head_dim = head_dim;
  a.scale = scale;
  a.kv_len = kv_len;
  a.splits = splits;
  a.out = out;
  a.part = k->ws;
  a.counter = k->ws_counter;
  return gb_attn_launch(a, (cudaStream_t)stream, false);
}

// ---- AttnDecode without allocation ------------------------------------------
namespace {
// The slice partials and per-KV-head counters of gb_gpu_attn_decode_noalloc
// live in file-scope device arrays of fixed size (4 MiB of partials, 256
// counters), one copy per device, shared by every call on that device.
constexpr size_t kNoAllocPartFloats = (size_t)1 << 20;
constexpr int kNoAllocHeads = 256;
constexpr int kNoAllocDevices = 64;
__device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
__device__ __align__(256) unsigned g_noalloc_counter[kNoAllocHeads];

struct NoAllocScratch {
  float *part = nullptr;
  unsigned *counter = nullptr;
};
NoAllocScratch g_noalloc[kNoAllocDevices];
std::mutex g_noalloc_mu;

// Addresses of the arrays on `device`, resolved once per device with that
// device current.
int noalloc_scratch(int device, NoAllocScratch *out) {
  if (device < 0 || device >= kNoAllocDevices)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode (no-alloc): device %d (0..%d)", device, kNoAllocDevices - 1);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocScratch &s = g_noalloc[device];
  if (!s.part) {
    int cur = 0;
    GB_CUDA(cudaGetDevice(&cur), "gpu: AttnDecode (no-alloc): current device");
    if (cur != device) GB_CUDA(cudaSetDevice(device), "gpu: AttnDecode (no-alloc): set device");
    void *part = nullptr, *counter = nullptr;
    cudaError_t e1 = cudaGetSymbolAddress(&part, g_noalloc_part);
    cudaError_t e2 = e1 == cudaSuccess ? cudaGetSymbolAddress(&counter, g_noalloc_counter) : e1;
    if (cur != device) cudaSetDevice(cur);
    GB_CUDA(e2, "gpu: AttnDecode (no-alloc): scratch address");
    s.part = (float *)part;
    s.counter = (unsigned *)counter;
  }
  *out = s;
  return GB_OK;
}

}  // namespace

int gb_gpu_attn_decode_noalloc(gb_kernels *k, void *stream, const float *q, const float *kcache,
                               const float *vcache, float *out, int kv_len, int n_heads, int n_kv,
                               int head_dim, float scale) {
  gb_clear_error();
  GB_NEED(k);
  if (kv_len <= 0) return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: kv_len %d", kv_len);
  if (n_kv <= 0 || n_heads % n_kv)
    return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: %d heads is not a multiple of %d KV heads", n_heads, n_kv);
  if (n_kv > kNoAllocHeads)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode (no-alloc): %d KV heads, at most %d", n_kv, kNoAllocHeads);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, k->device);
  int splits = (2 * sms + n_kv - 1) / n_kv;
  if (splits > 128) splits = 128;
  if (splits > kv_len) splits = kv_len;
  while ((kv_len + splits - 1) / splits > 2048) splits++;
  const int G = n_heads / n_kv;
  const size_t need = gb_attn_part_floats(n_kv, splits, G, head_dim);
  if (need > kNoAllocPartFloats)
    return gb_fail(GB_ERR_UNSUPPORTED,
                   "gpu: AttnDecode (no-alloc): %zu floats of slice partials needed, the static scratch holds %zu",
                   need, kNoAllocPartFloats);
  NoAllocScratch s;
  if (int rc = noalloc_scratch(k->device, &s)) return rc;
  // the counters must start at zero (each launch also leaves them at zero)
  GB_CUDA(cudaMemsetAsync(s.counter, 0, sizeof(unsigned) * (size_t)n_kv, (cudaStream_t)stream),
          "gpu: AttnDecode (no-alloc): clear counters");
  GbAttnArgs a;
  a.q = q;
  a.k = kcache;
  a.v = vcache;
  a.kv_f16 = 0;
  const long long kv_dim = (long long)n_kv * head_dim;
  a.k_sh = head_dim;
  a.k_sd = 4;
  a.k_st = kv_dim;
  a.v_sh = head_dim;
  a.v_st = kv_dim;
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.head_dim = head_dim;
  a.scale = scale;
  a.kv_len = kv_len;
  a.splits = splits;
  a.out = out;
  a.part = s.part;
  a.counter = s.counter;
  return gb_attn_launch(a, (cudaStream_t)stream, false);
}

int gb_gpu_matvec_f16(gb_kernels *k, void *stream, const uint16_t *w, const float *x, float *y,
                      int rows, int cols, int batch) {
  gb_clear_error();
  GB_NEED(k);
  if (rows <= 0 || batch <= 0) return GB_OK;
  matvec_dense_kernel<true><<<dim3((rows + 7) / 8, batch), 256, 0, (cudaStream_t)stream>>>(w, x, y, rows, cols);
  GB_CUDA(cudaGetLastError(), "gpu: MatVecF16");
  return GB_OK;
}

int gb_gpu_matvec_f32(gb_kernels *k, void *stream, const float *w, const float *x, float *y,
                      int rows, int cols, int batch) {
  gb_clear_error();
  GB_NEED(k);
  if (rows <= 0 || batch <= 0) return GB_OK;
  matvec_dense_kernel<false><<<dim3((rows + 7) / 8, batch), 256, 0, (cudaStream_t)stream>>>(w, x, y, rows, cols);
  GB_CUDA(cudaGetLastError(), "gpu: MatVecF32");
  return GB_OK;
}

// backend/gpu/gpu.go:137-153: type dispatch and the block-multiple check.
int gb_gpu_matvec_q(gb_kernels *k, void *stream, int typ, const uint8_t *w, const float *x,
                    float *y, int rows, int cols, int batch) {
  gb_clear_error();
  GB_NEED(k);
  const char *name;
  switch (typ) {
    case GB_T_Q4_0: name = "MatVecQ4_0"; break;
    case GB_T_Q4_K: name = "MatVecQ4K"; break;
    case GB_T_Q6_K: name = "MatVecQ6K"; break;
    default: return gb_fail(GB_ERR_UNSUPPORTED, "gpu: no matvec kernel for %s", type_name(typ));
  }
  if (cols % gb_block_size(typ) != 0)
    return gb_fail(GB_ERR_INVALID, "gpu: %s: %d columns is not a multiple of the block (%d)", name,
                   cols, gb_block_size(typ));
  if (rows <= 0 || batch <= 0) return GB_OK;
  matvec_q_raw_kernel<<<dim3((rows + 7) / 8, batch), 256, 0, (cudaStream_t)stream>>>(typ, w, x, y, rows, cols);
  GB_CUDA(cudaGetLastError(), name);
  return GB_OK;
}

int gb_gpu_ones(int n, float **out) {
  gb_clear_error();
  if (!out || n < 0) return gb_fail(GB_ERR_INVALID, "gpu: Ones: bad arguments");
  float *p = nullptr;
  GB_CUDA(cudaMalloc(&p, sizeof(float) * (size_t)(n > 0 ? n : 1)), "gpu: Ones");
  if (n > 0) {
    fill_kernel<<<blocks_for(n, 256), 256>>>(p, n, 1.f);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      cudaFree(p);
      return gb_cuda_fail(e, "gpu: Ones");
    }
  }
  *out = p;
  return GB_OK;
}

int gb_free(void *p) {
  gb_clear_error();
  if (p) GB_CUDA(cudaFree(p), "gpu: free");
  return GB_OK;
}

int gb_gpu_dequant_rows(gb_kernels *k, void *stream, int typ, const uint8_t *w, int rows, int cols,
                        int row0, int nrows, float *out) {
  gb_clear_error();
  GB_NEED(k);
  if (row0 < 0 || nrows < 0 || (long long)row0 + nrows > rows)
    return gb_fail(GB_ERR_INVALID, "quant: rows [%d, %d) outside the %d-row matrix", row0, row0 + nrows, rows);
  if (gb_block_size(typ) == 0) return gb_fail(GB_ERR_UNSUPPORTED, "quant: %s not supported", type_name(typ));
  if (cols % gb_block_size(typ))
    return gb_fail(GB_ERR_INVALID, "quant: %d elements is not a multiple of the %s block (%d)", cols,
                   type_name(typ), gb_block_size(typ));
  if (nrows <= 0) return GB_OK;
  dequant_rows_kernel<<<blocks_for((long long)nrows * cols, 256), 256, 0, (cudaStream_t)stream>>>(
      typ, w, cols, row0, nrows, out);
  GB_CUDA(cudaGetLastError(), "gpu: dequant");
  return GB_OK;
}

int gb_gpu_argmax(gb_kernels *k, void *stream, const float *x, int n, int32_t *out) {
  gb_clear_error();
  GB_NEED(k);
  if (n <= 0) return gb_fail(GB_ERR_INVALID, "gpu: argmax: empty vector");
  argmax_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, n, out);
  GB_CUDA(cudaGetLastError(), "gpu: argmax");
  return GB_OK;
}

int gb_gpu_peer_resid(gb_kernels *k, void *stream, int world, const float *const *bufs,
                      const unsigned *const *flags, const unsigned *step, int slot, int dim, float *x, int n,
                      float *ssq, unsigned wait_limit, unsigned *status) {
  gb_clear_error();
  GB_NEED(k);
  if (world < 1 || world > 32 || !bufs || !flags || !step || slot < 0 || !x || !ssq || n <= 0 || n % 32 ||
      n > dim)
    return gb_fail(GB_ERR_INVALID, "gpu: peer residual: bad arguments");
  GbPeer p;
  p.world = world;
  p.dim = dim;
  p.bufs = bufs;
  p.flags = flags;
  p.epoch = step;
  p.wait_limit = wait_limit ? wait_limit : p.wait_limit;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned *word = status ? status : k->status;
  int rc = gb_peer_resid_launch(p, slot, x, n, ssq, word, st, false);
  if (rc || status) return rc;
  // no status word of the caller's: wait for the call and report its outcome
  unsigned h = 0;
  GB_CUDA(cudaMemcpyAsync(&h, k->status, sizeof h, cudaMemcpyDeviceToHost, st), "gpu: peer residual");
  GB_CUDA(cudaStreamSynchronize(st), "gpu: peer residual");
  if (h) {
    GB_CUDA(cudaMemsetAsync(k->status, 0, sizeof h, st), "gpu: peer residual");
    GB_CUDA(cudaStreamSynchronize(st), "gpu: peer residual");
    return gb_fail(GB_ERR_TIMEOUT, "gpu: peer residual: a rank's flag did not arrive within %u polls", p.wait_limit);
  }
  return GB_OK;
}

int gb_gpu_peer_resid_tagged(gb_kernels *k, void *stream, int world, const unsigned long long *const *bufs,
                             const unsigned *step, int slot, int dim, float *x, int n, float *ssq,
                             unsigned wait_limit, unsigned *status) {
  gb_clear_error();
  GB_NEED(k);
  if (world < 1 || world > kGbMaxWorld || !bufs || !step || slot < 0 || !x || !ssq || n <= 0 || n % 32 || n > dim)
    return gb_fail(GB_ERR_INVALID, "gpu: peer residual: bad arguments");
  GbTagTable t = {};
  for (int q = 0; q < world; q++) {
    if (!bufs[q]) return gb_fail(GB_ERR_INVALID, "gpu: peer residual: rank %d has no buffer", q);
    t.w[q] = bufs[q];
  }
  const unsigned limit = wait_limit ? wait_limit : GbPeer().wait_limit;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned *word = status ? status : k->status;
  int rc = gb_peer_resid_tagged_launch(t, world, step, limit, slot, dim, x, n, ssq, word, st, false);
  if (rc || status) return rc;
  // no status word of the caller's: wait for the call and report its outcome
  unsigned h = 0;
  GB_CUDA(cudaMemcpyAsync(&h, k->status, sizeof h, cudaMemcpyDeviceToHost, st), "gpu: peer residual");
  GB_CUDA(cudaStreamSynchronize(st), "gpu: peer residual");
  if (h) {
    GB_CUDA(cudaMemsetAsync(k->status, 0, sizeof h, st), "gpu: peer residual");
    GB_CUDA(cudaStreamSynchronize(st), "gpu: peer residual");
    return gb_fail(GB_ERR_TIMEOUT, "gpu: peer residual: a rank's partial did not arrive within %u polls", limit);
  }
  return GB_OK;
}

int gb_gpu_sample(gb_kernels *k, void *stream, const float *logits, int n, const gb_sample_params *p,
                  const int32_t *recent, int n_recent, uint64_t counter, int32_t *out) {
  gb_clear_error();
  GB_NEED(k);
  if (!logits || !p || !out || n <= 0 || n_recent < 0 || (n_recent > 0 && !recent))
    return gb_fail(GB_ERR_INVALID, "gpu: sample: bad arguments");
  return gb_sample_launch(logits, n, p, nullptr, recent, n_recent, nullptr, nullptr, 0, counter, out, nullptr,
                          nullptr, (cudaStream_t)stream);
}

int gb_gpu_attn_decode_paged(gb_kernels *k, void *stream, const float *q, const void *k_pool, const void *v_pool,
                             int kv_f16, const int32_t *block_table, const int32_t *seq_lens, int batch,
                             int max_pages, int n_pages, int page_size, int n_heads, int n_kv, int head_dim,
                             float scale, float *out) {
  gb_clear_error();
  GB_NEED(k);
  if (batch < 0 || max_pages <= 0 || n_pages <= 0 || page_size <= 0 || !q || !k_pool || !v_pool || !block_table ||
      !seq_lens || !out)
    return gb_fail(GB_ERR_INVALID, "gpu: paged attention: bad arguments");
  if (n_kv <= 0 || n_heads % n_kv)
    return gb_fail(GB_ERR_INVALID, "gpu: paged attention: %d heads is not a multiple of %d KV heads", n_heads, n_kv);
  if (batch == 0) return GB_OK;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, k->device);
  // splits of each sequence's positions: about two CTAs per SM in all
  const long long max_chunks = ((long long)max_pages * page_size + 31) / 32;
  long long S = (2LL * sms + (long long)n_kv * batch - 1) / ((long long)n_kv * batch);
  if (S > max_chunks) S = max_chunks;
  if (S > 32) S = 32;
  if (S < 1) S = 1;
  const size_t need = gb_paged_part_floats(batch, n_kv, (int)S, n_heads / n_kv, head_dim);
  const size_t cnt = (size_t)batch * n_kv;
  if (need > k->pws_floats || cnt > k->pws_counters) {
    if (k->pws) cudaFree(k->pws);
    if (k->pws_counter) cudaFree(k->pws_counter);
    k->pws = nullptr;
    k->pws_counter = nullptr;
    k->pws_floats = k->pws_counters = 0;
    GB_CUDA(cudaMalloc(&k->pws, need * sizeof(float)), "gpu: paged attention: workspace");
    GB_CUDA(cudaMalloc(&k->pws_counter, cnt * sizeof(unsigned)), "gpu: paged attention: workspace");
    GB_CUDA(cudaMemsetAsync(k->pws_counter, 0, cnt * sizeof(unsigned), (cudaStream_t)stream),
            "gpu: paged attention: workspace");
    k->pws_floats = need;
    k->pws_counters = cnt;
  }
  return gb_attn_paged_launch(q, k_pool, v_pool, kv_f16, block_table, seq_lens, batch, max_pages, n_pages, page_size,
                              n_heads, n_kv, head_dim, scale, out, nullptr, k->pws, k->pws_counter, (int)S, nullptr,
                              (cudaStream_t)stream);
}

// model.Argmax, model/model.go:376.
// model.Argmax's rule: walking from index 0, an element replaces the best so
// far when it compares greater, so the first maximum wins, a NaN at index 0
// is returned and any later NaN is never taken. Two passes over the logits:
// the largest value (every comparison has the same "greater" form, so NaNs
// are skipped), then the first index holding it (== treats -0 and +0 alike,
// as the walk does). With SSE2 the first pass keeps 16 running maxima
// (MAXPS(a, m) is a > m ? a : m, NaN in a keeps m) and the second tests 16
// elements per step: ~17 us for 128256 logits where the walk took ~180 us.
int32_t gb_argmax(const float *logits, int64_t n) {
  if (n <= 0) return 0;
  const float x0 = logits[0];
  if (x0 != x0) return 0;
  float best = x0;
  int64_t i = 0, k = 0;
#if defined(__SSE2__) && !defined(__CUDA_ARCH__)
  __m128 m0 = _mm_set1_ps(x0), m1 = m0, m2 = m0, m3 = m0;
  for (; i + 16 <= n; i += 16) {
    m0 = _mm_max_ps(_mm_loadu_ps(logits + i), m0);
    m1 = _mm_max_ps(_mm_loadu_ps(logits + i + 4), m1);
    m2 = _mm_max_ps(_mm_loadu_ps(logits + i + 8), m2);
    m3 = _mm_max_ps(_mm_loadu_ps(logits + i + 12), m3);
  }
  float lanes[16];
  _mm_storeu_ps(lanes, m0);
  _mm_storeu_ps(lanes + 4, m1);
  _mm_storeu_ps(lanes + 8, m2);
  _mm_storeu_ps(lanes + 12, m3);
  for (int j = 0; j < 16; j++) best = lanes[j] > best ? lanes[j] : best;
#endif
  for (; i < n; i++) best = logits[i] > best ? logits[i] : best;
#if defined(__SSE2__) && !defined(__CUDA_ARCH__)
  const __m128 b4 = _mm_set1_ps(best);
  for (; k + 16 <= n; k += 16) {
    const __m128 c0 = _mm_or_ps(_mm_cmpeq_ps(_mm_loadu_ps(logits + k), b4), _mm_cmpeq_ps(_mm_loadu_ps(logits + k + 4), b4));
    const __m128 c1 =
        _mm_or_ps(_mm_cmpeq_ps(_mm_loadu_ps(logits + k + 8), b4), _mm_cmpeq_ps(_mm_loadu_ps(logits + k + 12), b4));
    if (_mm_movemask_ps(_mm_or_ps(c0, c1))) break;
  }
#endif
  for (; k < n; k++)
    if (logits[k] == best) return (int32_t)k;
  return 0;  // not reached: best is one of the values
}

}  // extern "C"
