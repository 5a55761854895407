// gb_sample.cu -- on-device token sampling: repetition penalty, temperature,
// top-k, top-p and a seeded counter-based draw, so that one int32 per token
// leaves the GPU (the reference picks greedily on the host with
// model.Argmax, cmd/gollama/run.go:124, model/model.go:376; sampling is its
// roadmap item "temperature, top-k, top-p, repetition penalty, seeded RNG").
//
// The rule, stated so that a host restatement reproduces every bit:
//  1. v_i = logits[i]; for every distinct id among the last `repeat_last_n`
//     context tokens: v = v <= 0 ? v*rp : v/rp (float32, rounded).
//  2. temperature <= 0 or top_k == 1: the token is the first maximum of v
//     (model.Argmax's rule). Otherwise s_i = v_i / temperature.
//  3. top_k <= 0 and top_p >= 1: every token is a candidate, in index order.
//     Else the candidates are the K = min(top_k > 0 ? top_k : 1024, 1024, n)
//     largest s by (value descending, index ascending), in that order.
//  4. e_i = exp(s_i - max s) with gb_exp_nonpos below; C_i = running sums in
//     the fixed association of the reduction written here (per-thread
//     chunks, then a Hillis-Steele scan over 1024 lanes).
//  5. top-p keeps the candidates up to the first c with C_c >= top_p*C_last.
//  6. u = splitmix64(seed, counter) in [0, 1) with 24 bits; the token is the
//     first candidate i <= c with C_i > u*C_c (the maximum if none is).
// Ordering keys make NaN the smallest value and -0 equal to +0.
#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr int kT = 1024;  // threads of the sampling CTA = candidate slots
constexpr int kMaxK = 1024;
static_assert(kMaxK == kT, "one candidate slot per thread");

// e^x for x <= 0, written from the mathematics rather than taken from a
// library: Cody-Waite reduction x = n ln2 + r with ln2 split as in Cephes
// (C1 = 355/512 exact, C2 = ln2 - C1), |r| <= ~0.35, e^r by its degree-7
// Taylor polynomial (truncation below 1e-8 relative), then the exact scale
// 2^n. Every operation is a single rounded float32 operation (fma where
// written), so the host restatement computes the same bits. x < -87 (and
// NaN) gives 0; results are never subnormal.
GB_DEV float gb_exp_nonpos(float x) {
  if (!(x >= -87.f)) return 0.f;
  const float n = rintf(__fmul_rn(x, 1.44269502f));
  float r = __fmaf_rn(-n, 0.693359375f, x);
  r = __fmaf_rn(-n, -2.12194440e-4f, r);
  float p = 1.98412698e-4f;  // 1/7!
  p = __fmaf_rn(p, r, 1.38888889e-3f);  // 1/6!
  p = __fmaf_rn(p, r, 8.33333333e-3f);  // 1/5!
  p = __fmaf_rn(p, r, 4.16666667e-2f);  // 1/4!
  p = __fmaf_rn(p, r, 1.66666667e-1f);  // 1/3!
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.f);
  p = __fmaf_rn(p, r, 1.f);
  return __fmul_rn(p, __uint_as_float((uint32_t)((int)n + 127) << 23));
}

// splitmix64 (Steele, Lea and Flood 2014) of seed + (counter+1)*golden, top 24 bits.
GB_DEV float gb_uniform24(unsigned long long seed, unsigned long long counter) {
  unsigned long long z = seed + (counter + 1ull) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(uint32_t)(z >> 40) * (1.f / 16777216.f);
}

// Order-preserving key of a float: larger value, larger key; NaN lowest.
GB_DEV uint32_t okey(float f) {
  if (f != f) return 0u;
  uint32_t b = __float_as_uint(f);
  if ((b << 1) == 0u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
GB_DEV float okey_value(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k); }

struct SArgs {
  const float *logits;
  int n;
  GbSampleParams p;
  const GbSampleParams *pd;   // device copy of the parameters (graph replays), or null
  const int32_t *recent;      // explicit context ids (device), or null
  int n_recent;
  const int32_t *fed;         // model: token fed at each position (device [max_len])
  const int32_t *pos;         // model: current position (device): the window end and the counter
  int max_len;
  unsigned long long counter;
  int32_t *out;               // the token (device)
  int32_t *gen;               // model: gen[pos] = the token
  unsigned *err;
};

// Value of element i after the penalty (and the temperature when t > 0).
GB_DEV float sval(const float *lg, int i, const uint32_t *bm, float rp, float t) {
  float v = __ldcg(lg + i);
  if (bm && ((bm[i >> 5] >> (i & 31)) & 1u)) v = v <= 0.f ? __fmul_rn(v, rp) : __fdiv_rn(v, rp);
  if (t > 0.f) v = __fdiv_rn(v, t);
  return v;
}

// Inclusive Hillis-Steele scan of a[kT] in place: a[i] = a[i-d] + a[i] for
// d = 1, 2, 4, ... (the association the host restatement repeats).
template <class V>
GB_DEV void hs_scan(V *a) {
  const int t = threadIdx.x;
  for (int d = 1; d < kT; d <<= 1) {
    V v = a[t];
    if (t >= d) v = a[t - d] + v;
    __syncthreads();
    a[t] = v;
    __syncthreads();
  }
}

GB_DEV unsigned long long block_max_u64(unsigned long long v, unsigned long long *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

GB_DEV int block_min_int(int v, int *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(kT, 1) sample_kernel(const SArgs a) {
  extern __shared__ uint32_t bm[];  // penalty bitmap, one bit per token
  __shared__ unsigned long long ck[kT];
  __shared__ float cum[kT];
  __shared__ int iscan[kT];
  __shared__ unsigned hist[256];
  __shared__ unsigned long long red64[32];
  __shared__ int redi[32];
  __shared__ uint32_t sh_prefix;
  __shared__ int sh_remaining, sh_c, sh_pick;
  const int t = threadIdx.x, n = a.n;
  const GbSampleParams p = a.pd ? *a.pd : a.p;
  unsigned long long counter = a.counter;
  int posv = 0;
  if (a.pos) {
    posv = *a.pos;
    posv = posv < 0 ? 0 : posv >= a.max_len ? a.max_len - 1 : posv;
    counter = (unsigned long long)posv;
  }

  // 1. the penalty set as a bitmap (duplicates collapse)
  const bool pen = p.repeat_penalty != 1.f && p.repeat_last_n > 0;
  if (pen) {
    for (int w = t; w < (n + 31) >> 5; w += kT) bm[w] = 0u;
    __syncthreads();
    int lo, hi;
    const int32_t *ids;
    if (a.fed) {
      ids = a.fed;
      hi = posv + 1;
    } else {
      ids = a.recent;
      hi = a.n_recent;
    }
    lo = hi - p.repeat_last_n;
    if (lo < 0) lo = 0;
    for (int q = lo + t; q < hi; q += kT) {
      int id = ids[q];
      if (id >= 0 && id < n) atomicOr(&bm[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
  }
  const uint32_t *bmp = pen ? bm : nullptr;
  const float rp = p.repeat_penalty;
  const bool greedy = !(p.temperature > 0.f) || p.top_k == 1;
  const float temp = greedy ? 0.f : p.temperature;

  // first maximum of the (penalised, tempered) values: the greedy token,
  // the shift of the exponentials and the fallback pick
  unsigned long long best = 0ull;
  for (int i = t; i < n; i += kT) {
    unsigned long long k = ((unsigned long long)okey(sval(a.logits, i, bmp, rp, temp)) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    best = k > best ? k : best;
  }
  best = block_max_u64(best, red64);
  const int arg = (int)(0xFFFFFFFFu - (uint32_t)best);
  const float mx = okey_value((uint32_t)(best >> 32));
  int pick = arg;
  const float u = gb_uniform24(p.seed, counter);
  const int C = (n + kT - 1) / kT;  // per-thread chunk of the index-ordered passes
  const int c0 = min(n, t * C), c1 = min(n, c0 + C);

  if (greedy) {
    // pick = arg
  } else if (p.top_k <= 0 && !(p.top_p < 1.f)) {
    // 3a. every token, in index order
    float local = 0.f;
    for (int i = c0; i < c1; i++) local = __fadd_rn(local, gb_exp_nonpos(__fsub_rn(sval(a.logits, i, bmp, rp, temp), mx)));
    cum[t] = local;
    __syncthreads();
    hs_scan(cum);
    const float total = cum[kT - 1];
    const float target = __fmul_rn(u, total);
    float acc = t ? cum[t - 1] : 0.f;
    int hit = 0x7FFFFFFF;
    for (int i = c0; i < c1; i++) {
      acc = __fadd_rn(acc, gb_exp_nonpos(__fsub_rn(sval(a.logits, i, bmp, rp, temp), mx)));
      if (acc > target) {
        hit = i;
        break;
      }
    }
    hit = block_min_int(hit, redi);
    if (hit != 0x7FFFFFFF) pick = hit;
  } else {
    // 3b. the K largest: radix select of the K-th key, 8 bits a pass
    int K = (p.top_k <= 0 || p.top_k > kMaxK) ? kMaxK : p.top_k;
    if (K > n) K = n;
    uint32_t prefix = 0u, mask = 0u;
    int remaining = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = t; b < 256; b += kT) hist[b] = 0u;
      __syncthreads();
      for (int i0 = 0; i0 < n; i0 += kT) {  // warp-uniform trip count
        const int i = i0 + t;
        const uint32_t k = i < n ? okey(sval(a.logits, i, bmp, rp, temp)) : 0u;
        const bool in = i < n && (k & mask) == prefix;
        const unsigned dig = (k >> shift) & 255u;
        // lanes of a warp that fall in one bin add once
        const unsigned act = __ballot_sync(0xffffffffu, in);
        if (in) {
          const unsigned same = __match_any_sync(act, dig);
          if ((__ffs(same) - 1) == (t & 31)) atomicAdd(&hist[dig], (unsigned)__popc(same));
        }
      }
      __syncthreads();
      if (t < 32) {
        // lane l owns bins 255-8l .. 248-8l; find the bin holding the remaining-th largest
        unsigned g = 0;
        for (int j = 0; j < 8; j++) g += hist[255 - 8 * t - j];
        unsigned inc = g;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          unsigned v = __shfl_up_sync(0xffffffffu, inc, o);
          if (t >= o) inc += v;
        }
        const unsigned excl = inc - g;
        const bool mine = excl < (unsigned)remaining && inc >= (unsigned)remaining;
        if (mine) {
          unsigned cacc = excl;
          for (int j = 0; j < 8; j++) {
            const int b = 255 - 8 * t - j;
            if (cacc + hist[b] >= (unsigned)remaining) {
              sh_prefix = prefix | ((uint32_t)b << shift);
              sh_remaining = remaining - (int)cacc;
              break;
            }
            cacc += hist[b];
          }
        }
      }
      __syncthreads();
      prefix = sh_prefix;
      remaining = sh_remaining;
      mask |= 255u << shift;
    }
    const uint32_t kth = prefix;
    const int need_eq = remaining, cnt_gt = K - need_eq;
    // gather in index order: keys above kth, then the first need_eq equal to it
    int ngt = 0, neq = 0;
    for (int i = c0; i < c1; i++) {
      const uint32_t k = okey(sval(a.logits, i, bmp, rp, temp));
      ngt += k > kth;
      neq += k == kth;
    }
    iscan[t] = ngt;
    __syncthreads();
    hs_scan(iscan);
    int gpos = iscan[t] - ngt;
    __syncthreads();
    iscan[t] = neq;
    __syncthreads();
    hs_scan(iscan);
    int epos = iscan[t] - neq;
    ck[t] = 0ull;
    __syncthreads();
    for (int i = c0; i < c1; i++) {
      const uint32_t k = okey(sval(a.logits, i, bmp, rp, temp));
      int slot = -1;
      if (k > kth) slot = gpos++;
      else if (k == kth && epos < need_eq) slot = cnt_gt + epos++;
      if (slot >= 0) ck[slot] = ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)i);
    }
    // bitonic sort, descending by (value, -index)
    for (int size = 2; size <= kT; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        __syncthreads();
        const int j = t ^ stride;
        if (j > t) {
          const unsigned long long x = ck[t], y = ck[j];
          const bool up = (t & size) == 0;
          if ((x < y) == up) {
            ck[t] = y;
            ck[j] = x;
          }
        }
      }
    __syncthreads();
    const float v0 = okey_value((uint32_t)(ck[0] >> 32));
    cum[t] = t < K ? gb_exp_nonpos(__fsub_rn(okey_value((uint32_t)(ck[t] >> 32)), v0)) : 0.f;
    __syncthreads();
    hs_scan(cum);
    if (t == 0) sh_c = K - 1;
    __syncthreads();
    if (p.top_p < 1.f) {
      const float thr = __fmul_rn(p.top_p, cum[kT - 1]);
      if (cum[t] >= thr && (t == 0 || cum[t - 1] < thr)) sh_c = t;
      __syncthreads();
    }
    const int c = min(sh_c, K - 1);
    const float target = __fmul_rn(u, cum[c]);
    if (t == 0) sh_pick = 0;
    __syncthreads();
    if (t <= c && cum[t] > target && (t == 0 || cum[t - 1] <= target)) sh_pick = t;
    __syncthreads();
    pick = (int)(0xFFFFFFFFu - (uint32_t)ck[sh_pick]);
  }
  if (t == 0) {
    *a.out = pick;
    if (a.gen) a.gen[posv] = pick;
  }
}

}  // namespace

int gb_sample_smem_bytes(int n) { return ((n + 31) / 32) * 4; }

int gb_sample_launch(const float *logits, int n, const GbSampleParams *p_host, const GbSampleParams *p_dev,
                     const int32_t *recent, int n_recent, const int32_t *fed, const int32_t *pos, int max_len,
                     unsigned long long counter, int32_t *out, int32_t *gen, unsigned *err, cudaStream_t st) {
  if (n <= 0 || n > kSampleMaxVocab) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: sample: vocabulary of %d", n);
  const int smem = gb_sample_smem_bytes(n);
  if (smem > 48 * 1024)  // the bitmap of a vocabulary above 393216 ids
    GB_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "gpu: sample");
  SArgs a{};
  a.logits = logits;
  a.n = n;
  if (p_host) a.p = *p_host;
  a.pd = p_dev;
  a.recent = recent;
  a.n_recent = n_recent;
  a.fed = fed;
  a.pos = pos;
  a.max_len = max_len;
  a.counter = counter;
  a.out = out;
  a.gen = gen;
  a.err = err;
  sample_kernel<<<1, kT, smem, st>>>(a);
  GB_CUDA(cudaGetLastError(), "gpu: sample");
  return GB_OK;
}
