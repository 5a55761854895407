// gb_paged.cu -- decode attention over a paged KV cache for a batch of
// sequences (the reference's roadmap "Paged KV cache plus continuous
// batching ... the attention kernel reads through a page table",
// ROADMAP.md:197-202; per sequence the arithmetic of cpu.AttnDecode,
// backend/cpu/cpu.go:140-168, whose GPU twin is (*Kernels).AttnDecode,
// backend/gpu/gpu.go:118).
//
// Pool layout: k_pool / v_pool = [n_pages][n_kv][page_size][head_dim]
// (binary16 or float32); sequence b's logical page i lives in physical page
// block_table[b * max_pages + i]; its keys are positions [0, seq_lens[b]).
// One CTA per (KV head, sequence, split of the pages): eight warps take the
// split's 32-position chunks in turn, lane = position for the scores of the
// group's query heads (q in shared memory), then lane = 4 dimensions for
// P V; online softmax per warp, the warps merged in shared memory, and the
// splits of a sequence merged by the last CTA to finish (a counter per
// (sequence, KV head)). float32 arithmetic throughout.
#include <math.h>

#include <algorithm>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr int kPW = 8;          // warps per CTA
constexpr int kPMaxG = 8;       // query heads per KV head
constexpr int kPMaxHD = 128;    // head_dim
constexpr int kPDL = kPMaxHD / 32;
// 16-byte pieces a thread moves per chunk: 2 x 32 rows of up to 512 bytes
constexpr int kPFetch = 2 * 32 * (kPMaxHD * 4 / 16) / (kPW * 32);

template <bool F16>
GB_DEV float ld_kv(const void *pool, size_t i) {
  if constexpr (F16) return gb_half_to_float(((const uint16_t *)pool)[i]);
  else return ((const float *)pool)[i];
}

// Eight consecutive elements (index a multiple of 8) as float.
template <bool F16>
GB_DEV void ld8(const void *pool, size_t i, float *o) {
  if constexpr (F16) {
    const uint4 u = *(const uint4 *)((const uint16_t *)pool + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      o[2 * j] = gb_half_to_float((uint16_t)(w[j] & 0xFFFF));
      o[2 * j + 1] = gb_half_to_float((uint16_t)(w[j] >> 16));
    }
  } else {
    const float4 x = *(const float4 *)((const float *)pool + i), y = *(const float4 *)((const float *)pool + i + 4);
    o[0] = x.x, o[1] = x.y, o[2] = x.z, o[3] = x.w, o[4] = y.x, o[5] = y.y, o[6] = y.z, o[7] = y.w;
  }
}

struct PagedArgs {
  const float *q;           // [B][n_heads][hd]
  const void *k_pool, *v_pool;
  const int32_t *block_table;  // [B][max_pages]
  const int32_t *seq_lens;     // [B]
  const int32_t *groups;       // null, or [n_groups + 1] first rows of the row groups
  int B, n_heads, n_kv, hd, page_size, max_pages, n_pages;
  float scale;
  float *out;               // [B][n_heads][hd]
  __half *out16;            // or, when set, the output in binary16
  float *part;              // [B][n_kv][S][G][hd + 2] split partials (m, l, acc)
  unsigned *counter;        // [B][n_kv], zero between launches
  int S;                    // splits of the pages
  unsigned *err;
};

// Bytes of one staged K or V row: the row plus 16 bytes, so that lanes
// reading rows 16 bytes at a time fall on distinct banks.
template <bool F16>
constexpr int row_stride(int hd) {
  return hd * (F16 ? 2 : 4) + 16;
}

// The chunk [ch*32, ch*32+32) of K and V into registers: thread t moves the
// 16-byte pieces t, t + blockDim, ... of the chunk's 2 x 32 rows (positions
// at or past L, and pieces past the rows, as zeros).
template <bool F16>
GB_DEV void chunk_fetch(const PagedArgs &a, int b, int h, int ch, int L, uint4 (&reg)[kPFetch]) {
  const int ppr = a.hd * (F16 ? 2 : 4) / 16;  // pieces per row
  const int32_t *table = a.block_table + (size_t)b * a.max_pages;
#pragma unroll
  for (int i = 0; i < kPFetch; i++) {
    const int piece = (int)threadIdx.x + i * kPW * 32, kv = piece / (32 * ppr), rem = piece % (32 * ppr);
    const int j = rem / ppr, pc = rem % ppr, p = ch * 32 + j;
    reg[i] = make_uint4(0, 0, 0, 0);
    if (kv < 2 && p < L) {
      int phys = table[p / a.page_size];
      if (phys < 0 || phys >= a.n_pages) {
        if (a.err) atomicOr(a.err, GB_DEVERR_POS);
        phys = 0;
      }
      const size_t row = (((size_t)phys * a.n_kv + h) * a.page_size + p % a.page_size) * a.hd;
      const uint8_t *pool = (const uint8_t *)(kv ? a.v_pool : a.k_pool) + row * (F16 ? 2 : 4);
      reg[i] = __ldcg((const uint4 *)pool + pc);
    }
  }
}
template <bool F16>
GB_DEV void chunk_store(const PagedArgs &a, const uint4 (&reg)[kPFetch], uint8_t *ks, uint8_t *vs) {
  const int ppr = a.hd * (F16 ? 2 : 4) / 16, rs = row_stride<F16>(a.hd);
#pragma unroll
  for (int i = 0; i < kPFetch; i++) {
    const int piece = (int)threadIdx.x + i * kPW * 32, kv = piece / (32 * ppr), rem = piece % (32 * ppr);
    if (kv < 2) *(uint4 *)((kv ? vs : ks) + (size_t)(rem / ppr) * rs + (rem % ppr) * 16) = reg[i];
  }
}

// One CTA per (KV head, row group, split of the positions). A row group is
// one row, or (with `groups`) up to kPW / G consecutive rows of one sequence
// that share its page table; warp w owns query head h*G + w % G of the
// group's row w / G. The split's 32-position chunks (up to the group's
// longest row) go through shared memory one after another, the next chunk's
// loads in flight while this one is used, so a group's rows read each chunk
// once: lane = position for the scores (masked at the warp's own row
// length), lane = dimensions lane + 32 i for P V, an online softmax per warp.
// One split writes the output itself; with several, each writes (m, l, acc)
// per row and the last to finish merges them.
template <bool F16>
__global__ void __launch_bounds__(kPW * 32) attn_paged_kernel(const PagedArgs a) {
  const int h = blockIdx.x, sp = blockIdx.z;
  const int G = a.n_heads / a.n_kv, hd = a.hd, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = a.groups ? a.groups[blockIdx.y] : (int)blockIdx.y;
  const int nr = a.groups ? a.groups[blockIdx.y + 1] - r0 : 1;
  const int rr = warp / G, g = warp % G, b = r0 + rr;  // this warp's row and head
  const bool active = rr < nr;
  constexpr int RS = row_stride<F16>(kPMaxHD);
  __shared__ float qs[kPW][kPMaxHD];
  __shared__ __align__(16) uint8_t ks[32 * RS], vs[32 * RS];
  __shared__ unsigned last;
  int Lmax = 0;
  for (int r = 0; r < nr; r++) Lmax = max(Lmax, a.seq_lens[r0 + r]);
  const int L = active ? a.seq_lens[b] : 0;
  for (int i = threadIdx.x; i < nr * G * hd; i += blockDim.x) {
    const int w = i / hd, d = i % hd;  // warp slot w = row * G + head
    qs[w][d] = a.q[((size_t)(r0 + w / G) * a.n_heads + (size_t)h * G + w % G) * hd + d];
  }
  const int nchunk = (Lmax + 31) / 32;
  const int c0 = (int)((long long)nchunk * sp / a.S), c1 = (int)((long long)nchunk * (sp + 1) / a.S);
  const int rs = row_stride<F16>(hd), DL = hd / 32;
  float m = -INFINITY, l = 0.f, acc[kPDL];
#pragma unroll
  for (int d = 0; d < kPDL; d++) acc[d] = 0.f;
  uint4 reg[kPFetch];
  if (c0 < c1) chunk_fetch<F16>(a, r0, h, c0, Lmax, reg);
  for (int ch = c0; ch < c1; ch++) {
    __syncthreads();  // the previous chunk is used up (and q is in place)
    chunk_store<F16>(a, reg, ks, vs);
    __syncthreads();
    if (ch + 1 < c1) chunk_fetch<F16>(a, r0, h, ch + 1, Lmax, reg);
    if (active && ch * 32 < L) {
      const int p = ch * 32 + lane;
      const bool in = p < L;
      float sc = 0.f;
      const uint8_t *kr = ks + (size_t)lane * rs;
      for (int d0 = 0; d0 < hd; d0 += F16 ? 8 : 4) {
        const uint4 u = *(const uint4 *)(kr + (F16 ? d0 * 2 : d0 * 4));
        float kv[8];
        if constexpr (F16) {
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; e++) {
            kv[2 * e] = gb_half_to_float((uint16_t)(w[e] & 0xFFFF));
            kv[2 * e + 1] = gb_half_to_float((uint16_t)(w[e] >> 16));
          }
        } else {
          kv[0] = __uint_as_float(u.x), kv[1] = __uint_as_float(u.y), kv[2] = __uint_as_float(u.z),
          kv[3] = __uint_as_float(u.w);
        }
#pragma unroll
        for (int e = 0; e < (F16 ? 8 : 4); e++) sc = fmaf(qs[warp][d0 + e], kv[e], sc);
      }
      const float sv = in ? sc * a.scale : -INFINITY;
      const float mn = fmaxf(m, gb_warp_max(sv));
      const float alpha = expf(m - mn), pe = in ? expf(sv - mn) : 0.f;
      l = l * alpha + gb_warp_sum(pe);
      m = mn;
#pragma unroll
      for (int d = 0; d < kPDL; d++) acc[d] *= alpha;
      const int jn = min(32, L - ch * 32);
      for (int j = 0; j < jn; j++) {
        const float pj = __shfl_sync(0xffffffffu, pe, j);
        const uint8_t *vr = vs + (size_t)j * rs;
#pragma unroll
        for (int d = 0; d < kPDL; d++)
          if (d < DL) {
            const float v = F16 ? gb_half_to_float(((const uint16_t *)vr)[lane + 32 * d])
                                : ((const float *)vr)[lane + 32 * d];
            acc[d] = fmaf(pj, v, acc[d]);
          }
      }
    }
  }
  if (a.S == 1) {
    if (active)
#pragma unroll
      for (int d = 0; d < kPDL; d++)
        if (d < DL) {
          const float o = l > 0.f ? acc[d] / l : 0.f;
          const size_t idx = ((size_t)b * a.n_heads + (size_t)h * G + g) * hd + lane + 32 * d;
          if (a.out16) a.out16[idx] = __float2half_rn(o);
          else a.out[idx] = o;
        }
    return;
  }
  if (active) {
    float *dst = a.part + (((size_t)b * a.n_kv + h) * a.S + sp) * G * (hd + 2);
#pragma unroll
    for (int d = 0; d < kPDL; d++)
      if (d < DL) dst[(size_t)g * (hd + 2) + 2 + lane + 32 * d] = acc[d];
    if (lane == 0) {
      dst[(size_t)g * (hd + 2)] = m;
      dst[(size_t)g * (hd + 2) + 1] = l;
    }
  }
  // the last split of (row group, KV head) merges the splits (in split order)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(a.counter + (size_t)r0 * a.n_kv + h, 1u) == (unsigned)(a.S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = threadIdx.x; i < nr * G * hd; i += blockDim.x) {
    const int row = r0 + i / (G * hd), gg = (i / hd) % G, d = i % hd;
    const float *src = a.part + ((size_t)row * a.n_kv + h) * a.S * G * (hd + 2);
    float M = -INFINITY;
    for (int s2 = 0; s2 < a.S; s2++) M = fmaxf(M, __ldcg(src + ((size_t)s2 * G + gg) * (hd + 2)));
    float Lsum = 0.f, A = 0.f;
    for (int s2 = 0; s2 < a.S; s2++) {
      const float *ps = src + ((size_t)s2 * G + gg) * (hd + 2);
      const float ms = __ldcg(ps);
      const float f = ms == -INFINITY ? 0.f : expf(ms - M);
      Lsum += __ldcg(ps + 1) * f;
      A += __ldcg(ps + 2 + d) * f;
    }
    const float o = Lsum > 0.f ? A / Lsum : 0.f;
    const size_t idx = ((size_t)row * a.n_heads + (size_t)h * G + gg) * hd + d;
    if (a.out16) a.out16[idx] = __float2half_rn(o);
    else a.out[idx] = o;
  }
  if (threadIdx.x == 0) a.counter[(size_t)r0 * a.n_kv + h] = 0u;  // ready for the next launch
}

// ---- batched decode helpers (one row per sequence) --------------------------

// RoPE of row t's q and k at position pos[t] (the model's float64 angle
// table, cpu.RoPE's rotation), q to q_out[t], k and v (binary16) into the
// pools at row pos % page_size of page table[t][pos / page_size].
__global__ void rope_kv_paged_kernel(const float *qkv, int q_rows, int kv_rows, int hd, const double *rope_cs,
                                     const int32_t *pos, const int32_t *table, int max_pages, int page_size,
                                     int n_pages, int max_len, float *q_out, uint16_t *kpool, uint16_t *vpool,
                                     unsigned *err) {
  const int t = blockIdx.x, p = pos[t];
  const int n_kv = kv_rows / hd;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;  // this thread's item
  const bool ok = p >= 0 && p < max_len && p / page_size < max_pages;
  int page = ok ? table[(size_t)t * max_pages + p / page_size] : -1;
  if (!ok || page < 0 || page >= n_pages) {
    if (threadIdx.x == 0 && err) atomicOr(err, GB_DEVERR_POS);
    return;
  }
  const int off = p % page_size;
  const float *row = qkv + (size_t)t * (q_rows + 2 * kv_rows);
  const double *cs = rope_cs + (size_t)p * hd;
  const int pairs = (q_rows + kv_rows) / 2;
  if (i < pairs + kv_rows) {
    if (i < pairs) {
      const int r = 2 * i, rr = r < q_rows ? r : r - q_rows, jj = (rr % hd) >> 1;
      const double c = cs[2 * jj], sn = cs[2 * jj + 1], x0 = row[r], x1 = row[r + 1];
      const float o0 = (float)__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, sn));
      const float o1 = (float)__dadd_rn(__dmul_rn(x0, sn), __dmul_rn(x1, c));
      if (r < q_rows) {
        q_out[(size_t)t * q_rows + r] = o0;
        q_out[(size_t)t * q_rows + r + 1] = o1;
      } else {
        const int h = rr / hd, d = rr % hd;
        const size_t idx = (((size_t)page * n_kv + h) * page_size + off) * hd + d;
        kpool[idx] = gb_float_to_half_rn(o0);
        kpool[idx + 1] = gb_float_to_half_rn(o1);
      }
    } else {
      const int rr = i - pairs, h = rr / hd, d = rr % hd;
      vpool[(((size_t)page * n_kv + h) * page_size + off) * hd + d] = gb_float_to_half_rn(row[q_rows + kv_rows + rr]);
    }
  }
}

__global__ void f32_to_f16_kernel(const float *x, __half *y, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

// First maximum of each row (model.Argmax's rule; NaN never wins).
// Order key of element i with value v: larger value first, then lower index;
// 0 for NaN (never wins) and the same key for +0 and -0.
GB_DEV unsigned long long argmax_key(float v, int i) {
  if (v != v) return 0ull;
  uint32_t b = __float_as_uint(v);
  if ((b << 1) == 0u) b = 0u;
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)i);
}

__global__ void argmax_rows_kernel(const float *x, int n, int32_t *out) {
  const float *row = x + (size_t)blockIdx.x * n;
  unsigned long long best = 0ull;
  if ((n & 3) == 0 && ((uintptr_t)row & 15) == 0) {  // four elements a load, eight loads in flight
    const float4 *r4 = (const float4 *)row;
    const int n4 = n >> 2;
#pragma unroll 8
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = r4[i];
      const unsigned long long k0 = argmax_key(v.x, 4 * i), k1 = argmax_key(v.y, 4 * i + 1);
      const unsigned long long k2 = argmax_key(v.z, 4 * i + 2), k3 = argmax_key(v.w, 4 * i + 3);
      const unsigned long long a = k0 > k1 ? k0 : k1, c = k2 > k3 ? k2 : k3, m = a > c ? a : c;
      best = m > best ? m : best;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long key = argmax_key(row[i], i);
      best = key > best ? key : best;
    }
  }
  __shared__ unsigned long long red[32];
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, best, o);
    best = w > best ? w : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    out[blockIdx.x] = best ? (int32_t)(0xFFFFFFFFu - (uint32_t)best) : 0;
  }
}

}  // namespace

size_t gb_paged_part_floats(int B, int n_kv, int S, int G, int hd) {
  return (size_t)B * n_kv * S * G * (hd + 2);
}

int gb_attn_paged_group_rows(int G) { return G >= 1 && G <= kPW ? kPW / G : 1; }

int gb_attn_paged_launch(const float *q, const void *k_pool, const void *v_pool, int kv_f16, const int32_t *block_table,
                         const int32_t *seq_lens, int B, int max_pages, int n_pages, int page_size, int n_heads,
                         int n_kv, int hd, float scale, float *out, __half *out16, float *part, unsigned *counter,
                         int S, unsigned *err, cudaStream_t st, const int32_t *groups, int n_groups) {
  if (B <= 0) return GB_OK;
  if (n_kv <= 0 || n_heads % n_kv || n_heads / n_kv > kPMaxG || hd % 32 || hd > kPMaxHD || page_size <= 0)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: paged attention: %d heads, %d KV heads, head_dim %d, page %d", n_heads,
                   n_kv, hd, page_size);
  PagedArgs a;
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.block_table = block_table;
  a.seq_lens = seq_lens;
  a.groups = groups;
  a.B = B;
  a.n_heads = n_heads;
  a.n_kv = n_kv;
  a.hd = hd;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.n_pages = n_pages;
  a.scale = scale;
  a.out = out;
  a.out16 = out16;
  a.part = part;
  a.counter = counter;
  a.S = S;
  a.err = err;
  const dim3 grid((unsigned)n_kv, (unsigned)(groups ? n_groups : B), (unsigned)S);
  if (kv_f16)
    attn_paged_kernel<true><<<grid, kPW * 32, 0, st>>>(a);
  else
    attn_paged_kernel<false><<<grid, kPW * 32, 0, st>>>(a);
  GB_CUDA(cudaGetLastError(), "gpu: paged attention");
  return GB_OK;
}

int gb_rope_kv_paged_launch(const float *qkv, int T, int q_rows, int kv_rows, int hd, const double *rope_cs,
                            const int32_t *pos, const int32_t *table, int max_pages, int page_size, int n_pages,
                            int max_len, float *q_out, uint16_t *kpool, uint16_t *vpool, unsigned *err,
                            cudaStream_t st) {
  if (T <= 0) return GB_OK;
  const unsigned items = (unsigned)((q_rows + kv_rows) / 2 + kv_rows);
  rope_kv_paged_kernel<<<dim3((unsigned)T, (items + 255) / 256), 256, 0, st>>>(qkv, q_rows, kv_rows, hd, rope_cs, pos, table, max_pages, page_size, n_pages,
                                          max_len, q_out, kpool, vpool, err);
  GB_CUDA(cudaGetLastError(), "engine: RoPE/KV append");
  return GB_OK;
}

int gb_f32_to_f16_launch(const float *x, __half *y, size_t n, cudaStream_t st) {
  if (!n) return GB_OK;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  f32_to_f16_kernel<<<blocks, 256, 0, st>>>(x, y, n);
  GB_CUDA(cudaGetLastError(), "engine: convert");
  return GB_OK;
}

int gb_argmax_rows_launch(const float *x, int rows, int n, int32_t *out, cudaStream_t st) {
  if (rows <= 0) return GB_OK;
  argmax_rows_kernel<<<rows, 1024, 0, st>>>(x, n, out);
  GB_CUDA(cudaGetLastError(), "engine: argmax");
  return GB_OK;
}
