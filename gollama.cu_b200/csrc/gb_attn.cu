// gb_attn.cu -- single-token attention (decode) as split-K flash decoding.
//
// Replaces kernels.AttnDecode (kernels/attention.go:15-60), whose one block per
// query head re-reads K once per head of a GQA group and is limited by a
// kv_len*4-byte score row in shared memory. Here one CTA serves a whole GQA
// group (all query heads of one KV head) over one slice of the positions,
// so K and V are read from HBM exactly once per token; slices are merged by
// the last CTA of each KV head with the log-sum-exp rule. Math is float32
// with float32 accumulators (the reference's cpu.AttnDecode accumulates in
// float64; tolerances cover the difference).
//
// Cache layouts are described by strides. The per-op API reads the
// reference's [kv_len][n_kv*head_dim] float32 caches. The model's caches are
// head-major: K as [head][head_dim/V][max_len][V] (V = 16 bytes of elements,
// so a position's 16-byte chunks of one dim range are contiguous across
// positions); V as [head][max_len][head_dim] for float32 caches and in the
// K layout for fp16 caches (the tensor-core kernel reads both as 8x8 tiles).
#include <math.h>
#include <stdlib.h>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <bool F16>
struct Chunk;
template <>
struct Chunk<true> {  // 8 halves
  static constexpr int V = 8;
  static GB_DEV void load(const void *base, long long off, float *out) {
    uint4 u = __ldg((const uint4 *)((const uint16_t *)base + off));
    unpack(u, out);
  }
  static GB_DEV void load_shared(const uint8_t *p, float *out) { unpack(*(const uint4 *)p, out); }
  static GB_DEV void unpack(uint4 u, float *out) {
    const __half2 *h = (const __half2 *)&u;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 f = __half22float2(h[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Chunk<false> {  // 4 floats
  static constexpr int V = 4;
  static GB_DEV void load(const void *base, long long off, float *out) {
    float4 f = __ldg((const float4 *)((const float *)base + off));
    out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
  }
  static GB_DEV void load_shared(const uint8_t *p, float *out) {
    float4 f = *(const float4 *)p;
    out[0] = f.x; out[1] = f.y; out[2] = f.z; out[3] = f.w;
  }
};

template <bool F16>
GB_DEV float vload(const void *base, long long off) {
  if (F16) return gb_half_to_float(((const uint16_t *)base)[off]);
  return ((const float *)base)[off];
}

// ---- slice partials and their merge -----------------------------------------
// A slice partial per (KV head, slice, group head g) is a row of HD + 4
// floats: the unnormalised output o[HD], the running max m, the sum l and two
// pad floats that keep rows 16-byte aligned for float4 loads.
constexpr int part_stride(int hd) { return hd + 4; }

// Shared-memory floats merge_slices needs: weights [S][8], 1/L [8], one
// float4 per thread.
__host__ __device__ constexpr int merge_floats(int S, int nthr) { return ((8 * S + 8 + 3) & ~3) + 4 * nthr; }

// Merge the S slice partials of KV head h into out with the
// log-sum-exp rule: out = sum_j exp(m_j - M) o_j / sum_j exp(m_j - M) l_j.
// Called by every thread of the head's last CTA. The slice weights come from
// one warp per group head (lanes over slices); the weighted sums are spread
// over all threads as float4 columns x slice groups and added in a fixed
// order, so the result is deterministic. The partials were written by other
// CTAs and are read from L2, where each dependent access costs a round trip
// of about a microsecond: every thread issues its loads -- the (m, l) pairs
// and up to kMergeBatch of its o columns -- before any arithmetic needs them.
constexpr int kMergeBatch = 16;

template <int HD>
GB_DEV void merge_slices(const GbAttnArgs &a, int h, int S, int G, float *ms, int nthr) {
  constexpr int PS = part_stride(HD);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *wgt = ms, *linv = ms + 8 * S;
  float4 *red4 = (float4 *)(ms + ((8 * S + 8 + 3) & ~3));
  const float *pb = a.part + (size_t)h * S * G * PS;
  const int NV = G * HD / 4, ngrp = nthr / NV;  // NV <= 256 <= nthr
  const bool mine = tid < ngrp * NV;
  const int v = tid % NV, grp = tid / NV, g = v / (HD / 4), d = (v % (HD / 4)) * 4;
  // 1. loads: this thread's first batch of o columns, and (m, l) of the slices
  float4 xb[kMergeBatch];
  int nb = 0;
  if (mine) {
#pragma unroll
    for (int q = 0; q < kMergeBatch; q++) {
      const int j = grp + q * ngrp;
      if (j < S) {
        xb[q] = __ldcg((const float4 *)(pb + ((size_t)j * G + g) * PS + d));
        nb = q + 1;
      }
    }
  }
  if (warp < G && S > 128) {  // more slices than the fast path holds: two passes over L2
    float M = -INFINITY;
    for (int j = lane; j < S; j += 32) M = fmaxf(M, __ldcg(pb + ((size_t)j * G + warp) * PS + HD));
    M = gb_warp_max(M);
    float L = 0.f;
    for (int j = lane; j < S; j += 32) {
      const float2 ml = __ldcg((const float2 *)(pb + ((size_t)j * G + warp) * PS + HD));
      const float w = ml.x == -INFINITY ? 0.f : expf(ml.x - M);
      wgt[j * 8 + warp] = w;
      L += ml.y * w;
    }
    L = gb_warp_sum(L);
    if (lane == 0) linv[warp] = 1.f / L;
  } else if (warp < G) {
    float2 ml[4];  // S <= 128 slices: at most 4 per lane
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int j = lane + 32 * q;
      ml[q] = j < S ? __ldcg((const float2 *)(pb + ((size_t)j * G + warp) * PS + HD)) : make_float2(-INFINITY, 0.f);
    }
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < 4; q++) M = fmaxf(M, ml[q].x);
    M = gb_warp_max(M);
    float L = 0.f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int j = lane + 32 * q;
      const float w = ml[q].x == -INFINITY ? 0.f : expf(ml[q].x - M);
      if (j < S) wgt[j * 8 + warp] = w;
      L += ml[q].y * w;
    }
    L = gb_warp_sum(L);
    if (lane == 0) linv[warp] = 1.f / L;
  }
  __syncthreads();
  // 2. weighted sums in slice order: the loaded batch, then any further batches
  if (mine) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int base = 0;; base += kMergeBatch) {
#pragma unroll
      for (int q = 0; q < kMergeBatch; q++) {
        if (q < nb) {
          const float w = wgt[(grp + (base + q) * ngrp) * 8 + g];
          acc.x = fmaf(xb[q].x, w, acc.x);
          acc.y = fmaf(xb[q].y, w, acc.y);
          acc.z = fmaf(xb[q].z, w, acc.z);
          acc.w = fmaf(xb[q].w, w, acc.w);
        }
      }
      if (grp + (base + kMergeBatch) * ngrp >= S) break;
      nb = 0;
#pragma unroll
      for (int q = 0; q < kMergeBatch; q++) {
        const int j = grp + (base + kMergeBatch + q) * ngrp;
        if (j < S) {
          xb[q] = __ldcg((const float4 *)(pb + ((size_t)j * G + g) * PS + d));
          nb = q + 1;
        }
      }
    }
    red4[tid] = acc;
  }
  __syncthreads();
  if (tid < NV) {
    float4 o = red4[tid];
    for (int gi = 1; gi < ngrp; gi++) {
      const float4 x = red4[gi * NV + tid];
      o.x += x.x;
      o.y += x.y;
      o.z += x.z;
      o.w += x.w;
    }
    const float li = linv[tid / (HD / 4)];
    o = make_float4(o.x * li, o.y * li, o.z * li, o.w * li);
    *(float4 *)(a.out + (size_t)h * G * HD + (size_t)tid * 4) = o;
  }
}

template <int GM, int HD, bool F16>
__global__ void __launch_bounds__(kThreads) attn_kernel(const GbAttnArgs a, int chunk_cap) {
  extern __shared__ __align__(16) float sm[];
  constexpr int V = Chunk<F16>::V;
  constexpr int DPL = HD / 32;  // dims per lane in P.V
  const int h = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int G = a.n_heads / a.n_kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *qs = sm;                      // [GM][HD]
  float *ps = qs + GM * HD;            // [GM][chunk_cap]
  float *red = ps + GM * chunk_cap;    // [kWarps][GM][HD]
  __shared__ float mx[GM], sum[GM], wred[kWarps][GM];
  __shared__ int last;

  gb_grid_dep_wait();  // q and the position come from the preceding kernel
  int kv_len = a.kv_len_pos ? (*a.kv_len_pos + 1) : a.kv_len;
  if (a.max_len > 0 && (kv_len < 1 || kv_len > a.max_len)) {
    if (tid == 0 && a.err) atomicOr(a.err, GB_DEVERR_POS);
    kv_len = kv_len < 1 ? 1 : a.max_len;
  }
  const int t0 = (int)((long long)kv_len * s / S), t1 = (int)((long long)kv_len * (s + 1) / S);
  const int nt = t1 - t0;

  for (int i = tid; i < G * HD; i += kThreads) qs[i] = a.q[(size_t)h * G * HD + i];
  __syncthreads();

  // scores: one thread per position, all G heads of the group
  float lmax[GM];
#pragma unroll
  for (int g = 0; g < GM; g++) lmax[g] = -INFINITY;
  const char *kb = (const char *)a.k;
  for (int t = t0 + tid; t < t1; t += kThreads) {
    float dot[GM];
#pragma unroll
    for (int g = 0; g < GM; g++) dot[g] = 0.f;
#pragma unroll 4
    for (int dc = 0; dc < HD / V; dc++) {
      float kv[V];
      Chunk<F16>::load(a.k, (long long)h * a.k_sh + (long long)dc * a.k_sd + (long long)t * a.k_st, kv);
#pragma unroll
      for (int g = 0; g < GM; g++) {
        if (g < G) {
          const float *qg = qs + g * HD + dc * V;
#pragma unroll
          for (int j = 0; j < V; j++) dot[g] = fmaf(qg[j], kv[j], dot[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < GM; g++) {
      if (g < G) {
        float sc = dot[g] * a.scale;
        ps[g * chunk_cap + (t - t0)] = sc;
        lmax[g] = fmaxf(lmax[g], sc);
      }
    }
  }
  (void)kb;
  // block max per head
#pragma unroll
  for (int g = 0; g < GM; g++) {
    float v = gb_warp_max(lmax[g]);
    if (lane == 0) wred[warp][g] = v;
  }
  __syncthreads();
  if (tid < GM) {
    float v = -INFINITY;
    for (int w = 0; w < kWarps; w++) v = fmaxf(v, wred[w][tid]);
    mx[tid] = v;
  }
  __syncthreads();
  float lsum[GM];
#pragma unroll
  for (int g = 0; g < GM; g++) lsum[g] = 0.f;
  for (int t = tid; t < nt; t += kThreads) {
#pragma unroll
    for (int g = 0; g < GM; g++) {
      if (g < G) {
        float e = expf(ps[g * chunk_cap + t] - mx[g]);
        ps[g * chunk_cap + t] = e;
        lsum[g] += e;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GM; g++) {
    float v = gb_warp_sum(lsum[g]);
    if (lane == 0) wred[warp][g] = v;
  }
  __syncthreads();
  if (tid < GM) {
    float v = 0.f;
    for (int w = 0; w < kWarps; w++) v += wred[w][tid];
    sum[tid] = v;
  }

  // P.V: warp w takes positions w, w+8, ...; lane owns DPL consecutive dims
  float acc[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; g++)
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[g][j] = 0.f;
  for (int t = warp; t < nt; t += kWarps) {
    long long vo = (long long)h * a.v_sh + (long long)(t0 + t) * a.v_st + lane * DPL;
    float vv[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) vv[j] = vload<F16>(a.v, vo + j);
#pragma unroll
    for (int g = 0; g < GM; g++) {
      if (g < G) {
        float p = ps[g * chunk_cap + t];
#pragma unroll
        for (int j = 0; j < DPL; j++) acc[g][j] = fmaf(p, vv[j], acc[g][j]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GM; g++)
#pragma unroll
    for (int j = 0; j < DPL; j++) red[(warp * GM + g) * HD + lane * DPL + j] = acc[g][j];
  __syncthreads();

  // this slice's partial: o[g][d] (unnormalised), m_g, l_g
  constexpr int PS = part_stride(HD);
  float *part = a.part + ((size_t)h * S + s) * G * PS;
  for (int i = tid; i < G * HD; i += kThreads) {
    int g = i / HD, d = i % HD;
    float o = 0.f;
    for (int w = 0; w < kWarps; w++) o += red[(w * GM + g) * HD + d];
    part[g * PS + d] = o;
  }
  if (tid < G) {
    part[tid * PS + HD] = mx[tid];
    part[tid * PS + HD + 1] = sum[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counter[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  merge_slices<HD>(a, h, S, G, sm, kThreads);  // the dynamic buffer is free now
  if (tid == 0) a.counter[h] = 0u;
  gb_grid_dep_launch();
}

// The model's head-major caches: flash decoding with a TMA ring. A CTA owns
// one KV head and one slice of the positions and walks the slice in
// sub-chunks of SUB = 256/GM positions. For every sub-chunk the K rows (HD/V
// contiguous runs of SUB*16 bytes) and the V rows (one run) arrive by 1-D TMA
// bulk copies into a ring of NSTAGE shared-memory stages, so the next
// sub-chunks stream in while this one is computed; the softmax is carried
// online (running max and sum per head). Sub-chunks that do not hold the new
// position are requested before waiting on the kernel that wrote it.
constexpr int kStages = 3;

template <int GM, int HD, bool F16>
struct Flash {
  static constexpr int V = Chunk<F16>::V;
  static constexpr int ESZ = F16 ? 2 : 4;
  static constexpr int SUB = kThreads / GM;            // positions per sub-chunk
  static constexpr int KBYTES = SUB * HD * ESZ;        // K (and V) bytes of a full sub-chunk
  static constexpr int STAGE = 2 * KBYTES;
  static constexpr int DPT = GM * HD / kThreads;       // output dims per thread in P.V
  static constexpr size_t smem() {
    return (size_t)kStages * STAGE + sizeof(float) * ((size_t)GM * HD + (size_t)GM * SUB);
  }
};

template <int GM, int HD, bool F16>
__global__ void __launch_bounds__(kThreads) attn_flash_kernel(const GbAttnArgs a) {
  using FL = Flash<GM, HD, F16>;
  constexpr int V = FL::V, ESZ = FL::ESZ, SUB = FL::SUB, DPT = FL::DPT;
  extern __shared__ __align__(128) uint8_t smb[];
  float *qs = (float *)(smb + (size_t)kStages * FL::STAGE);  // [GM][HD]
  float *sc = qs + GM * HD;                                 // [GM][SUB] scores, then probabilities
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ float m_run[GM], l_run[GM], alpha[GM], wred[kThreads / 32];
  __shared__ int last;
  const int h = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int G = a.n_heads / a.n_kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  gb_grid_dep_launch();  // one CTA per SM: the next kernel fits beside this one
  int kv_len = *a.kv_len_pos + 1;
  const bool bad = kv_len < 1 || kv_len > a.max_len;
  if (bad) kv_len = kv_len < 1 ? 1 : a.max_len;
  const int t0 = (int)((long long)kv_len * s / S), t1 = (int)((long long)kv_len * (s + 1) / S);
  const int nsub = (t1 - t0 + SUB - 1) / SUB;
  const long long kbase = (long long)h * a.k_sh, vbase = (long long)h * a.v_sh;
  auto issue = [&](int k) {  // sub-chunk k into stage k % kStages (thread 0)
    const int p0 = t0 + k * SUB, nk = min(SUB, t1 - p0);
    uint8_t *st = smb + (size_t)(k % kStages) * FL::STAGE;
    gb_mbar_expect_tx(&bars[k % kStages], (uint32_t)(2 * nk * HD * ESZ));
    for (int dc = 0; dc < HD / V; dc++)
      gb_bulk_g2s(st + (size_t)dc * SUB * 16, (const uint8_t *)a.k + (kbase + (long long)dc * a.k_sd + (long long)p0 * V) * ESZ,
                  (uint32_t)(nk * 16), &bars[k % kStages]);
    gb_bulk_g2s(st + FL::KBYTES, (const uint8_t *)a.v + (vbase + (long long)p0 * HD) * ESZ, (uint32_t)(nk * HD * ESZ),
                &bars[k % kStages]);
  };
  // the sub-chunk holding position kv_len-1 is written by the preceding kernel
  auto is_new = [&](int k) { return t0 + (k + 1) * SUB >= kv_len; };
  int issued = 0;
  if (tid == 0) {
    for (int i = 0; i < kStages; i++) gb_mbar_init(&bars[i], 1);
    gb_mbar_fence_init();
    while (issued < nsub && issued < kStages && !is_new(issued)) issue(issued++);
  }
  gb_grid_dep_wait();  // q and the new K/V row come from the preceding kernel
  if (tid == 0) {
    if (bad && a.err) atomicOr(a.err, GB_DEVERR_POS);
    gb_fence_proxy_async_global();  // the new row was written by generic stores
    while (issued < nsub && issued < kStages) issue(issued++);
  }
  if (tid < GM) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
  }
  for (int i = tid; i < G * HD; i += kThreads) qs[i] = a.q[(size_t)h * G * HD + i];
  __syncthreads();
  issued = __shfl_sync(0xffffffffu, issued, 0);  // thread 0's count (warp 0), then shared below
  __shared__ int issued_s;
  if (tid == 0) issued_s = issued;
  __syncthreads();
  issued = issued_s;

  const int qk_t = tid % SUB, qk_g = tid / SUB;                    // QK: one (position, head) per thread
  const int pv_g = tid / (HD / DPT), pv_d = (tid % (HD / DPT)) * DPT;  // P.V: DPT dims of one head
  float acc[DPT];
#pragma unroll
  for (int j = 0; j < DPT; j++) acc[j] = 0.f;
  bool ok = true;
  for (int k = 0; k < nsub; k++) {
    const int p0 = t0 + k * SUB, nk = min(SUB, t1 - p0);
    const uint8_t *st = smb + (size_t)(k % kStages) * FL::STAGE;
    ok = gb_mbar_wait(&bars[k % kStages], (uint32_t)((k / kStages) & 1)) && ok;
    // scores
    float sv = -INFINITY;
    if (ok && qk_g < G && qk_t < nk) {
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;  // four independent FMA chains
#pragma unroll
      for (int dc = 0; dc < HD / V; dc++) {
        float kv[V];
        Chunk<F16>::load_shared(st + ((size_t)dc * SUB + qk_t) * 16, kv);
        const float4 *qg = (const float4 *)(qs + qk_g * HD + dc * V);
#pragma unroll
        for (int j4 = 0; j4 < V / 4; j4++) {
          const float4 qv = qg[j4];
          d0 = fmaf(qv.x, kv[4 * j4], d0);
          d1 = fmaf(qv.y, kv[4 * j4 + 1], d1);
          d2 = fmaf(qv.z, kv[4 * j4 + 2], d2);
          d3 = fmaf(qv.w, kv[4 * j4 + 3], d3);
        }
      }
      sv = ((d0 + d1) + (d2 + d3)) * a.scale;
    }
    // running max per head: the SUB threads of a head are SUB/32 whole warps
    float wm = gb_warp_max(sv);
    if (lane == 0) wred[warp] = wm;
    __syncthreads();
    if (tid < GM) {
      float m = -INFINITY;
      for (int w = tid * (SUB / 32); w < (tid + 1) * (SUB / 32); w++) m = fmaxf(m, wred[w]);
      const float mn = fmaxf(m_run[tid], m);
      alpha[tid] = m_run[tid] == -INFINITY ? 0.f : expf(m_run[tid] - mn);
      m_run[tid] = mn;
    }
    __syncthreads();
    float pr = 0.f;
    if (qk_g < G && qk_t < nk && sv != -INFINITY) pr = expf(sv - m_run[qk_g]);
    if (qk_g < GM) sc[qk_g * SUB + qk_t] = pr;
    float ws = gb_warp_sum(pr);
    if (lane == 0) wred[warp] = ws;
    __syncthreads();
    if (tid < GM) {
      float sum = 0.f;
      for (int w = tid * (SUB / 32); w < (tid + 1) * (SUB / 32); w++) sum += wred[w];
      l_run[tid] = l_run[tid] * alpha[tid] + sum;
    }
    // P.V with the running rescale
    if (pv_g < G) {
      const float al = alpha[pv_g];
#pragma unroll
      for (int j = 0; j < DPT; j++) acc[j] *= al;
      const uint8_t *vs = st + FL::KBYTES;
      const float *pg = sc + pv_g * SUB;
      // two interleaved position streams: independent FMA chains
      float acc2[DPT];
#pragma unroll
      for (int j = 0; j < DPT; j++) acc2[j] = 0.f;
      auto vrow = [&](int t, float *vv) {
        if (F16) {
          if (DPT == 1) {
            vv[0] = gb_half_to_float(*(const uint16_t *)(vs + ((size_t)t * HD + pv_d) * ESZ));
          } else {
#pragma unroll
            for (int j = 0; j < DPT; j += 2) {
              const float2 f = __half22float2(*(const __half2 *)(vs + ((size_t)t * HD + pv_d + j) * ESZ));
              vv[j] = f.x;
              vv[j + 1] = f.y;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < DPT; j++) vv[j] = *(const float *)(vs + ((size_t)t * HD + pv_d + j) * ESZ);
        }
      };
      int t = 0;
#pragma unroll 2
      for (; t + 1 < nk; t += 2) {
        float v0[DPT], v1[DPT];
        vrow(t, v0);
        vrow(t + 1, v1);
        const float p0 = pg[t], p1 = pg[t + 1];
#pragma unroll
        for (int j = 0; j < DPT; j++) {
          acc[j] = fmaf(p0, v0[j], acc[j]);
          acc2[j] = fmaf(p1, v1[j], acc2[j]);
        }
      }
      if (t < nk) {
        float v0[DPT];
        vrow(t, v0);
#pragma unroll
        for (int j = 0; j < DPT; j++) acc[j] = fmaf(pg[t], v0[j], acc[j]);
      }
#pragma unroll
      for (int j = 0; j < DPT; j++) acc[j] += acc2[j];
    }
    __syncthreads();  // stage k is free; scores may be overwritten
    if (tid == 0 && issued < nsub) {
      gb_fence_proxy_async();
      issue(issued);
    }
    issued++;
    if (issued > nsub) issued = nsub;
  }
  if (!ok && tid == 0 && a.err) atomicOr(a.err, GB_DEVERR_TIMEOUT);

  // this slice's partial: o[g][d] (unnormalised), m_g, l_g
  constexpr int PS = part_stride(HD);
  float *part = a.part + ((size_t)h * S + s) * G * PS;
  if (pv_g < G) {
#pragma unroll
    for (int j = 0; j < DPT; j++) part[pv_g * PS + pv_d + j] = acc[j];
  }
  if (tid < G) {
    part[tid * PS + HD] = m_run[tid];
    part[tid * PS + HD + 1] = l_run[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counter[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // every issued stage has been waited on: the ring is free for the merge
  merge_slices<HD>(a, h, S, G, (float *)smb, kThreads);
  if (tid == 0) a.counter[h] = 0u;
}

template <int GM, int HD, bool F16>
int launch_flash(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  using FL = Flash<GM, HD, F16>;
  if (a.splits > 128) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: %d slices (128 at most)", a.splits);
  const size_t smem = FL::smem();
  static_assert(merge_floats(128, kThreads) * 4 <= kStages * FL::STAGE, "merge scratch exceeds the ring");
  static bool attr = false;
  if (!attr) {
    GB_CUDA(cudaFuncSetAttribute(attn_flash_kernel<GM, HD, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
            "gpu: AttnDecode: shared memory attribute");
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)a.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = pdl ? 1 : 0;
  GB_CUDA(cudaLaunchKernelEx(&cfg, attn_flash_kernel<GM, HD, F16>, a), "gpu: AttnDecode");
  return GB_OK;
}

// ---- flash decoding on tensor cores (fp16 caches) ---------------------------
// K and V are both cached as [head][HD/8][max_len][8] halves: a run of
// positions is HD/8 contiguous runs of 16 bytes per position for each of K
// and V. A producer warp streams sub-chunks of SUB = 16 * kMW positions
// through a ring of kMStages shared-memory stages with 1-D TMA bulk copies;
// each of the kMW consumer warps owns 16 positions of every sub-chunk and
// carries its own online softmax (running max and sum per head), so no block
// barrier runs inside the loop: a stage returns to the producer once its
// `empty` mbarrier has counted every consumer warp. After the loop the
// warps' states are combined in shared memory into the CTA's slice partial.
//
// Products on mma.sync m16n8k16 (fp16 inputs, fp32 accumulation), per warp
// and 16 positions:
//   S[16 x 16 pos]  = Qs[16 x HD] . K^T   (B fragments: K rows by ldmatrix)
//   O[16 x HD]     += Ps[16 x 16 pos] . V (B fragments: V rows by ldmatrix.trans)
// Rows 0..7 of Qs hold the group's query heads rounded to fp16 and rows 8..15
// the rounding residues, so rows g and g+8 of S add up to the score of head g
// with about 22 bits of q (fp16 x fp16 products are exact in fp32); rows 0..7
// of Ps hold p rounded to fp16 and rows 8..15 the residues. The accumulator
// layout of S is the A-operand layout of Ps, so p never leaves registers.
// The 16-byte rows of one 8x8 ldmatrix tile are contiguous in shared memory,
// so neither ldmatrix form has bank conflicts. GQA groups of up to 8 heads;
// smaller groups leave rows unused.
constexpr int kMW = 8;                     // consumer warps
constexpr int kMThreads = 32 * (kMW + 1);  // plus one producer warp
constexpr int kMStages = 3;

template <int HD>
struct MmaAttn {
  static constexpr int SUB = 16 * kMW;        // positions per sub-chunk
  static constexpr int HALF = SUB * HD * 2;   // K (or V) bytes of a full sub-chunk
  static constexpr int STAGE = 2 * HALF;
  static constexpr size_t smem() { return (size_t)kMStages * STAGE; }
  // after the loop: warp combine buffer [kMW][8][PS] in stage 0, merge scratch in stage 1
  static_assert(kMW * 8 * (HD + 4) * 4 <= STAGE, "combine buffer exceeds a stage");
  static_assert(merge_floats(128, kMThreads) * 4 <= STAGE, "merge scratch exceeds a stage");
};

template <int HD>
__global__ void __launch_bounds__(kMThreads, 1) attn_mma_kernel(const __grid_constant__ GbAttnArgs a) {
  using MA = MmaAttn<HD>;
  constexpr int SUB = MA::SUB, KS = HD / 16, NT = HD / 8, PS = part_stride(HD);
  static_assert(SUB == 128, "the tensor maps' box holds 128 positions");
  extern __shared__ __align__(128) uint8_t smb[];
  __shared__ __align__(8) uint64_t full[kMStages], empty[kMStages];
  __shared__ float wm[kMW][8], wl[kMW][8];
  __shared__ int last;
  const int h = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int G = a.n_heads / a.n_kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;

  gb_grid_dep_launch();
  // The position is written by the previous step's last kernel, which has
  // completed: only q and the new K/V row need the preceding kernel.
  int kv_len = *a.kv_len_pos + 1;
  const bool bad = kv_len < 1 || kv_len > a.max_len;
  if (bad) kv_len = kv_len < 1 ? 1 : a.max_len;
  // slice bounds on 32-position boundaries (the tensor maps address rows of 32 positions)
  const int t0 = s == 0 ? 0 : (int)((long long)kv_len * s / S) & ~31;
  const int t1 = s == S - 1 ? kv_len : (int)((long long)kv_len * (s + 1) / S) & ~31;
  const int nsub = (t1 - t0 + SUB - 1) / SUB;
  if (tid == 0) {
    for (int i = 0; i < kMStages; i++) {
      gb_mbar_init(&full[i], 1);
      gb_mbar_init(&empty[i], kMW);
    }
    gb_mbar_fence_init();
  }
  __syncthreads();

  bool ok = true;
  float m_run = -INFINITY, l_run = 0.f;
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  if (warp == kMW) {
    // producer: one lane issues every copy
    if (lane == 0) {
      if (bad && a.err) atomicOr(a.err, GB_DEVERR_POS);
      const uint8_t *kg = (const uint8_t *)a.k + (size_t)h * a.k_sh * 2;
      const uint8_t *vg = (const uint8_t *)a.v + (size_t)h * a.v_sh * 2;
      bool waited = false;
      for (int k = 0; k < nsub; k++) {
        const int st = k % kMStages;
        if (k >= kMStages) {
          if (!gb_mbar_wait(&empty[st], (uint32_t)((k / kMStages - 1) & 1))) {
            ok = false;
            break;
          }
          gb_fence_proxy_async();
        }
        // the sub-chunk holding position kv_len-1 is written by the preceding kernel
        if (!waited && t0 + (k + 1) * SUB >= kv_len) {
          gb_grid_dep_wait();
          gb_fence_proxy_async_global();  // the new row was written by generic stores
          waited = true;
        }
        const int p0 = t0 + k * SUB, nk = min(SUB, t1 - p0);
        uint8_t *sk = smb + (size_t)st * MA::STAGE, *sv = sk + MA::HALF;
        gb_mbar_expect_tx(&full[st], (uint32_t)(2 * NT * nk * 16));
        if (a.tmap && nk == SUB) {
          // a whole sub-chunk: one 4-D copy each of K and V lands as
          // [dim chunk][position][16 B], the layout the consumers read
          gb_tma_load_4d(sk, &a.tk, 0, p0 >> 5, 0, h, &full[st]);
          gb_tma_load_4d(sv, &a.tv, 0, p0 >> 5, 0, h, &full[st]);
          continue;
        }
        for (int dc = 0; dc < NT; dc++) {
          gb_bulk_g2s(sk + (size_t)dc * SUB * 16, kg + ((size_t)dc * a.k_sd + (size_t)p0 * 8) * 2,
                      (uint32_t)(nk * 16), &full[st]);
          gb_bulk_g2s(sv + (size_t)dc * SUB * 16, vg + ((size_t)dc * a.v_sd + (size_t)p0 * 8) * 2,
                      (uint32_t)(nk * 16), &full[st]);
        }
      }
    }
  } else {
    gb_grid_dep_wait();  // q comes from the preceding kernel
    // Qs rows gid (hi) and gid+8 (lo) as A fragments
    uint32_t qa[KS][4];
    {
      const float *qh = a.q + ((size_t)h * G + gid) * HD;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
          const int d = ks * 16 + 8 * r + 2 * tig;
          const float x0 = gid < G ? qh[d] : 0.f, x1 = gid < G ? qh[d + 1] : 0.f;
          split2(x0, x1, qa[ks][2 * r], qa[ks][2 * r + 1]);
        }
      }
    }
    const int wp0 = warp * 16, mi = lane >> 3, lr = lane & 7;
    for (int k = 0; k < nsub; k++) {
      const int st = k % kMStages;
      const int p0 = t0 + k * SUB, nv = min(SUB, t1 - p0) - wp0;  // valid positions of this warp
      ok = gb_mbar_wait(&full[st], (uint32_t)((k / kMStages) & 1)) && ok;
      const uint8_t *sk = smb + (size_t)st * MA::STAGE;
      uint8_t *sv = smb + (size_t)st * MA::STAGE + MA::HALF;
      if (ok && nv > 0) {
        if (nv < 16) {  // rows past the slice hold stale bytes: zero V there (p is 0, 0*NaN is not)
          const int nz = 16 - nv;
          for (int i = lane; i < nz * NT; i += 32)
            *(uint4 *)(sv + ((size_t)(i / nz) * SUB + wp0 + nv + i % nz) * 16) = make_uint4(0u, 0u, 0u, 0u);
          __syncwarp();
        }
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
          uint32_t b[4];
          ldsm_x4(b, sk + ((size_t)(2 * ks + (mi & 1)) * SUB + wp0 + (mi >> 1) * 8 + lr) * 16);
          mma16816(c0, qa[ks], b[0], b[1]);
          mma16816(c1, qa[ks], b[2], b[3]);
        }
        // this thread: head gid at local positions 2tig, 2tig+1, 8+2tig, 9+2tig
        float sc[4] = {c0[0] + c0[2], c0[1] + c0[3], c1[0] + c1[2], c1[1] + c1[3]};
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int lp = 2 * tig + (i & 1) + 8 * (i >> 1);
          sc[i] = lp < nv ? sc[i] * a.scale : -INFINITY;
          mx = fmaxf(mx, sc[i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m_run, mx);
        const float al = m_run == -INFINITY ? 0.f : expf(m_run - mn);
        float p[4], psum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          p[i] = sc[i] == -INFINITY ? 0.f : expf(sc[i] - mn);
          psum += p[i];
        }
        l_run = l_run * al + psum;
        m_run = mn;
        uint32_t pa[4];
        split2(p[0], p[1], pa[0], pa[1]);
        split2(p[2], p[3], pa[2], pa[3]);
#pragma unroll
        for (int n2 = 0; n2 < NT / 2; n2++) {
          uint32_t b[4];
          ldsm_x4_t(b, sv + ((size_t)(2 * n2 + (mi >> 1)) * SUB + wp0 + (mi & 1) * 8 + lr) * 16);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            o[2 * n2][j] *= al;
            o[2 * n2 + 1][j] *= al;
          }
          mma16816(o[2 * n2], pa, b[0], b[1]);
          mma16816(o[2 * n2 + 1], pa, b[2], b[3]);
        }
      }
      __syncwarp();
      if (lane == 0) gb_mbar_arrive(&empty[st]);
    }
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  }
  if (!ok && a.err) atomicOr(a.err, GB_DEVERR_TIMEOUT);

  // combine the warps' states into this slice's partial
  __syncthreads();  // every issued stage has been waited on: the ring is free
  if (warp < kMW && tig == 0) {
    wm[warp][gid] = m_run;
    wl[warp][gid] = l_run;
  }
  __syncthreads();
  float *red = (float *)smb;  // [kMW][8][PS]
  if (warp < kMW && gid < G) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMW; w++) M = fmaxf(M, wm[w][gid]);
    const float f = m_run == -INFINITY ? 0.f : expf(m_run - M);
    float *r = red + ((size_t)warp * 8 + gid) * PS;
#pragma unroll
    for (int n = 0; n < NT; n++)
      *(float2 *)(r + n * 8 + 2 * tig) = make_float2((o[n][0] + o[n][2]) * f, (o[n][1] + o[n][3]) * f);
  }
  __syncthreads();
  float *part = a.part + ((size_t)h * S + s) * G * PS;
  for (int i = tid; i < G * HD; i += kMThreads) {
    const int g = i / HD, d = i % HD;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kMW; w++) acc += red[((size_t)w * 8 + g) * PS + d];
    part[g * PS + d] = acc;
  }
  if (tid < G) {
    float M = -INFINITY, L = 0.f;
#pragma unroll
    for (int w = 0; w < kMW; w++) M = fmaxf(M, wm[w][tid]);
#pragma unroll
    for (int w = 0; w < kMW; w++)
      if (wm[w][tid] != -INFINITY) L += wl[w][tid] * expf(wm[w][tid] - M);
    part[tid * PS + HD] = M;
    part[tid * PS + HD + 1] = L;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counter[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  merge_slices<HD>(a, h, S, G, (float *)(smb + MA::STAGE), kMThreads);
  if (tid == 0) a.counter[h] = 0u;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <int HD>
int launch_mma(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  using MA = MmaAttn<HD>;
  if (a.splits > 128) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: %d slices (128 at most)", a.splits);
  const size_t smem = MA::smem();
  static bool attr = false;
  if (!attr) {
    GB_CUDA(cudaFuncSetAttribute(attn_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
            "gpu: AttnDecode: shared memory attribute");
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)a.splits);
  cfg.blockDim = dim3(kMThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = pdl ? 1 : 0;
  GB_CUDA(cudaLaunchKernelEx(&cfg, attn_mma_kernel<HD>, a), "gpu: AttnDecode");
  return GB_OK;
}

template <int GM, int HD, bool F16>
int launch_t(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.kv_len_pos && a.max_len > 0) {  // the model's head-major caches
    if constexpr (F16) {
      if (a.k_st != 8 || a.v_st != 8) return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: fp16 cache layout");
      return launch_mma<HD>(a, st, pdl);
    } else {
      if (a.k_st != 4 || a.v_st != HD) return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: fp32 cache layout");
      return launch_flash<GM, HD, false>(a, st, pdl);
    }
  }
  int cap_len = a.max_len > 0 ? a.max_len : a.kv_len;
  int chunk_cap = (cap_len + a.splits - 1) / a.splits + 1;
  size_t smem = sizeof(float) * ((size_t)GM * HD + (size_t)GM * chunk_cap + (size_t)kWarps * GM * HD);
  const size_t msmem = sizeof(float) * (size_t)merge_floats(a.splits, kThreads);
  if (smem < msmem) smem = msmem;
  if (a.splits > 128) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: %d slices (128 at most)", a.splits);
  if (smem > 200 * 1024) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: %d positions per slice", chunk_cap);
  static bool attr = false;
  if (!attr) {
    GB_CUDA(cudaFuncSetAttribute(attn_kernel<GM, HD, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
            "gpu: AttnDecode: shared memory attribute");
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)a.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = pdl ? 1 : 0;
  GB_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<GM, HD, F16>, a, chunk_cap), "gpu: AttnDecode");
  return GB_OK;
}

}  // namespace

// Slices per KV head for the model's caches of max_len positions: one CTA
// per SM (each streams its slice through a TMA ring that fills most of the
// SM's shared memory), at most 128 slices (the merge reads all of them) and
// at least 128 positions per slice at full length.
int gb_attn_splits(int n_kv, int max_len, int nsm) {
  int s = nsm / n_kv;
  if (s > 128) s = 128;
  int by_len = (max_len + 127) / 128;
  if (s > by_len) s = by_len;
  return s < 1 ? 1 : s;
}

size_t gb_attn_part_floats(int n_kv, int splits, int group, int head_dim) {
  return (size_t)n_kv * splits * group * part_stride(head_dim);
}

int gb_attn_launch(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.n_kv <= 0 || a.n_heads % a.n_kv != 0)
    return gb_fail(GB_ERR_INVALID, "gpu: AttnDecode: %d heads is not a multiple of %d KV heads", a.n_heads, a.n_kv);
  const int G = a.n_heads / a.n_kv;
  if (G > 8) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: GQA group %d above 8", G);
  const bool f16 = a.kv_f16 != 0;
  switch (a.head_dim) {
    case 64:
      if (G <= 4) return f16 ? launch_t<4, 64, true>(a, st, pdl) : launch_t<4, 64, false>(a, st, pdl);
      return f16 ? launch_t<8, 64, true>(a, st, pdl) : launch_t<8, 64, false>(a, st, pdl);
    case 128:
      if (G <= 4) return f16 ? launch_t<4, 128, true>(a, st, pdl) : launch_t<4, 128, false>(a, st, pdl);
      return f16 ? launch_t<8, 128, true>(a, st, pdl) : launch_t<8, 128, false>(a, st, pdl);
  }
  return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: head_dim %d (64 or 128 supported)", a.head_dim);
}

// Tensor maps of one layer's fp16 K and V caches. The cache is
// [kv_head][head_dim/8][max_len][8 halves]; as a 4-D tensor (innermost
// first) {256 = 32 positions x 8 halves, max_len/32, head_dim/8, n_kv} with
// byte strides {512, 16*max_len, 16*max_len*head_dim/8}. A box
// {256, 4, head_dim/8, 1} is one head's 128 positions (from a multiple of
// 32) of every 16-byte dim chunk, read as 512-byte rows, and lands in shared
// memory as [chunk][position][16 B] -- the stage layout of attn_mma_kernel.
// (A 16-byte innermost dimension would make the copy engine move 16-byte
// rows, slower than per-chunk 1-D copies; 256 is the largest box side.) The
// encoder comes from the driver
// through the runtime's entry-point query, so the library does not link
// libcuda.
int gb_attn_tensor_maps(const void *k, const void *v, int n_kv, int head_dim, int max_len, CUtensorMap *tk,
                        CUtensorMap *tv) {
  static EncodeTiledFn encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return gb_fail(GB_ERR_CUDA, "gpu: AttnDecode: cuTensorMapEncodeTiled unavailable");
    encode = (EncodeTiledFn)fn;
  }
  if (max_len < 128 || max_len % 32 || (head_dim != 64 && head_dim != 128))
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: no tensor map for max_len %d, head_dim %d", max_len, head_dim);
  const cuuint64_t dims[4] = {256, (cuuint64_t)(max_len / 32), (cuuint64_t)(head_dim / 8), (cuuint64_t)n_kv};
  const cuuint64_t strides[3] = {512, (cuuint64_t)max_len * 16, (cuuint64_t)max_len * 16 * (head_dim / 8)};
  const cuuint32_t box[4] = {256, 4, (cuuint32_t)(head_dim / 8), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const void *src[2] = {k, v};
  CUtensorMap *dst[2] = {tk, tv};
  for (int i = 0; i < 2; i++) {
    CUresult r = encode(dst[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void *>(src[i]), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return gb_fail(GB_ERR_CUDA, "gpu: AttnDecode: tensor map encode failed (%d)", (int)r);
  }
  return GB_OK;
}
