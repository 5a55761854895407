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
// Cache layouts are described by strides so that the same kernel reads the
// reference's [kv_len][n_kv*head_dim] float32 caches (per-op API) and the
// model's head-major caches: K as [head][head_dim/V][max_len][V] (V = 16
// bytes of elements, so one thread reads one position's 16-byte chunk and a
// warp reads 512 contiguous bytes), V as [head][max_len][head_dim].
#include <math.h>

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
  const int stride = HD + 2;
  float *part = a.part + ((size_t)h * S + s) * G * stride;
  for (int i = tid; i < G * HD; i += kThreads) {
    int g = i / HD, d = i % HD;
    float o = 0.f;
    for (int w = 0; w < kWarps; w++) o += red[(w * GM + g) * HD + d];
    part[g * stride + d] = o;
  }
  if (tid < G) {
    part[tid * stride + HD] = mx[tid];
    part[tid * stride + HD + 1] = sum[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counter[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();

  // merge the S slices of this KV head (fixed order: deterministic)
  const float *pbase = a.part + (size_t)h * S * G * stride;
  const int ngroups = G * HD / 32;
  for (int grp = warp; grp < ngroups; grp += kWarps) {
    int g = (grp * 32) / HD, d = (grp * 32) % HD + lane;
    float M = -INFINITY;
    for (int j = 0; j < S; j++) M = fmaxf(M, __ldcg(pbase + ((size_t)j * G + g) * stride + HD));
    float L = 0.f, O = 0.f;
    for (int j = 0; j < S; j++) {
      const float *pj = pbase + ((size_t)j * G + g) * stride;
      float m = __ldcg(pj + HD);
      float w = m == -INFINITY ? 0.f : expf(m - M);
      L += __ldcg(pj + HD + 1) * w;
      O += __ldcg(pj + d) * w;
    }
    float out = O / L;
    int oi = (h * G + g) * HD + d;
    a.out[oi] = out;
    if (a.out_pack.a) {
      GbXPack pk{a.out_pack.a, a.out_pack.b, a.out_pack.c, a.out_pack.s, a.out_pack.sum16, nullptr};
      gb_pack_group(pk, oi / 32, out);
    }
  }
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
  const int stride = HD + 2;
  float *part = a.part + ((size_t)h * S + s) * G * stride;
  if (pv_g < G) {
#pragma unroll
    for (int j = 0; j < DPT; j++) part[pv_g * stride + pv_d + j] = acc[j];
  }
  if (tid < G) {
    part[tid * stride + HD] = m_run[tid];
    part[tid * stride + HD + 1] = l_run[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counter[h], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();

  // merge the S slices of this KV head (fixed order: deterministic)
  const float *pbase = a.part + (size_t)h * S * G * stride;
  __shared__ float wgt[64 * 8], linv[GM];
  if (tid < G) {
    float M = -INFINITY;
    for (int j = 0; j < S; j++) M = fmaxf(M, __ldcg(pbase + ((size_t)j * G + tid) * stride + HD));
    float L = 0.f;
    for (int j = 0; j < S; j++) {
      const float m = __ldcg(pbase + ((size_t)j * G + tid) * stride + HD);
      const float w = m == -INFINITY ? 0.f : expf(m - M);
      wgt[j * GM + tid] = w;
      L += __ldcg(pbase + ((size_t)j * G + tid) * stride + HD + 1) * w;
    }
    linv[tid] = 1.f / L;
  }
  __syncthreads();
  for (int o = tid; o < G * HD; o += kThreads) {
    const int g = o / HD, d = o % HD;
    float O = 0.f;
#pragma unroll 8
    for (int j = 0; j < S; j++) O = fmaf(__ldcg(pbase + ((size_t)j * G + g) * stride + d), wgt[j * GM + g], O);
    const float out = O * linv[g];
    const int oi = (h * G + g) * HD + d;
    a.out[oi] = out;
    if (a.out_pack.a) {
      GbXPack pk{a.out_pack.a, a.out_pack.b, a.out_pack.c, a.out_pack.s, a.out_pack.sum16, nullptr};
      gb_pack_group(pk, oi / 32, out);
    }
  }
  if (tid == 0) a.counter[h] = 0u;
}

template <int GM, int HD, bool F16>
int launch_flash(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  using FL = Flash<GM, HD, F16>;
  if (a.splits > 64) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: AttnDecode: %d slices (64 at most)", a.splits);
  const size_t smem = FL::smem();
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

template <int GM, int HD, bool F16>
int launch_t(const GbAttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.kv_len_pos && a.max_len > 0 && a.k_st == Chunk<F16>::V && a.v_st == HD)
    return launch_flash<GM, HD, F16>(a, st, pdl);
  int cap_len = a.max_len > 0 ? a.max_len : a.kv_len;
  int chunk_cap = (cap_len + a.splits - 1) / a.splits + 1;
  size_t smem = sizeof(float) * ((size_t)GM * HD + (size_t)GM * chunk_cap + (size_t)kWarps * GM * HD);
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

// Slices per KV head for a cache of max_len positions: two CTAs per SM (each
// streams its slice through a TMA ring), at most 64 slices (the merge reads
// all of them) and at least 64 positions per slice at full length.
int gb_attn_splits(int n_kv, int max_len, int nsm) {
  int s = 2 * nsm / n_kv;
  if (s > 64) s = 64;
  int by_len = (max_len + 63) / 64;
  if (s > by_len) s = by_len;
  return s < 1 ? 1 : s;
}

size_t gb_attn_part_floats(int n_kv, int splits, int group, int head_dim) {
  return (size_t)n_kv * splits * group * (head_dim + 2);
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
