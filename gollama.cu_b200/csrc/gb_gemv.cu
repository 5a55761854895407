// gb_gemv.cu -- batch-1 quantized matrix-vector products on the tiled layout
// (gb_formats.h), with fused epilogues for the decode step.
//
// Replaces kernels.MatVecQ4_0 / MatVecQ4K / MatVecQ6K (kernels/quantmv.go:18-136)
// on the model path. Design:
//  * Work is the list of units (row-block, super-block); a row-block is one
//    32-row tile, or a gate/up tile pair for the SwiGLU epilogue. Every CTA
//    takes one contiguous range of units (stream-K over a persistent grid,
//    or one row-block per CTA for small matrices), so all SMs stay busy
//    whatever the matrix shape and no wave is partial.
//  * Units are contiguous in memory in that order, so a CTA's range is one
//    byte range. A producer warp streams it through a ring of shared-memory
//    stages of K units (tens of KB) with one 1-D TMA bulk copy per stage;
//    eight consumer warps decode the units round-robin and give each stage
//    back through an mbarrier. Lane l of a warp owns row l of the tile.
//  * The activation arrives as a limb pack (gb_device.cuh): three int8 limbs
//    per element, so the 4-bit / 6-bit quants meet the activation in dp4a
//    (4 products per instruction, exact int32 sums); float math is needed once
//    per 16- or 32-element sub-block for the ggml scales. A CTA stages only the
//    pack of the super-blocks its units touch.
//  * A row-block split between CTAs is finished by the CTA whose atomic
//    count completes it; it sums the partials in CTA order (deterministic)
//    and runs the epilogue. Counters are reset by that CTA, so the kernel can
//    be replayed from a CUDA graph.
//  * A CTA uses about half an SM, so under programmatic dependent launch the
//    next kernel's CTA fits beside it and streams its own weights during
//    this kernel's tail.
//  * One instantiation per (weight types, epilogue) keeps each kernel's code
//    small.
#include <math.h>
#include <stdlib.h>

#include <algorithm>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr float kL2 = 1.f / 64516.f;  // 1/254^2: limbs b, c are combined as 254*b + c

GB_DEV float byte_f(uint32_t w, int i) { return (float)((w >> (8 * i)) & 0xFFu); }

// ---- per-super-block decode + dot products. `st` is the sb-block in shared
// memory; xa/xb/xc are the limb planes (as 32-bit words) of the block's 256
// activation elements, xs the 8 group scales and xsum the 16 half-group sums.
template <int T>
GB_DEV float sb_dot(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xs, const float *xsum);

// Q4_K: quant/quant.go:97 layout; kernels/quantmv.go:66 factorisation
// sum = d*sum_j sc_j*(q.x)_j - dmin*sum_j m_j*(sum x)_j.
template <>
GB_DEV float sb_dot<GB_T_Q4_K>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  const uint4 h = u[lane];
  const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFFu));
  const float dmin = gb_half_to_float((uint16_t)(h.x >> 16));
  const uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
  const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  float tq = 0.f, tm = 0.f;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 q0 = u[(1 + 2 * c) * 32 + lane], q1 = u[(2 + 2 * c) * 32 + lane];
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint4 *pa = (const uint4 *)(xa + 16 * c), *pb = (const uint4 *)(xb + 16 * c),
                *pc = (const uint4 *)(xc + 16 * c);
    int A0 = 0, B0 = 0, C0 = 0, A1 = 0, B1 = 0, C1 = 0;
#pragma unroll
    for (int v = 0; v < 2; v++) {
      const uint4 la = pa[v], lb = pb[v], lc = pc[v], ha = pa[2 + v], hb = pb[2 + v], hc = pc[2 + v];
      const uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
                     c4[4] = {lc.x, lc.y, lc.z, lc.w};
      const uint32_t A4[4] = {ha.x, ha.y, ha.z, ha.w}, B4[4] = {hb.x, hb.y, hb.z, hb.w},
                     C4[4] = {hc.x, hc.y, hc.z, hc.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint32_t w = qw[4 * v + k];
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
        A0 = gb_dp4a_us(lo, a4[k], A0);
        B0 = gb_dp4a_us(lo, b4[k], B0);
        C0 = gb_dp4a_us(lo, c4[k], C0);
        A1 = gb_dp4a_us(hi, A4[k], A1);
        B1 = gb_dp4a_us(hi, B4[k], B1);
        C1 = gb_dp4a_us(hi, C4[k], C1);
      }
    }
    // sum q*x / s_g = A + (254 B + C)/254^2  (254 B + C < 2^24: exact in float)
    const float S0 = (float)A0 + (float)(254 * B0 + C0) * kL2;
    const float S1 = ((float)A1 + (float)(254 * B1 + C1) * kL2) * 0.0625f;
    const int j0 = 2 * c, j1 = 2 * c + 1;
    const float sc0 = byte_f(j0 < 4 ? sc03 : sc47, j0 & 3), sc1 = byte_f(j1 < 4 ? sc03 : sc47, j1 & 3);
    const float m0 = byte_f(j0 < 4 ? m03 : m47, j0 & 3), m1 = byte_f(j1 < 4 ? m03 : m47, j1 & 3);
    tq = fmaf(sc0, xs[j0] * S0, tq);
    tq = fmaf(sc1, xs[j1] * S1, tq);
    tm = fmaf(m0, xsum[2 * j0] + xsum[2 * j0 + 1], tm);
    tm = fmaf(m1, xsum[2 * j1] + xsum[2 * j1 + 1], tm);
  }
  return d * tq - dmin * tm;
}

// Q6_K: quant/quant.go:114 layout; y = d*sc*(q-32) over 16-element sub-blocks.
template <>
GB_DEV float sb_dot<GB_T_Q6_K>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  const uint4 scv = u[12 * 32 + lane];
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  const float d = gb_half_to_float(((const uint16_t *)(st + 13 * 512))[lane]);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 2; c++) {
    const uint4 l0 = u[(4 * c + 0) * 32 + lane], l1 = u[(4 * c + 1) * 32 + lane];
    const uint4 l2 = u[(4 * c + 2) * 32 + lane], l3 = u[(4 * c + 3) * 32 + lane];
    const uint4 h0 = u[(8 + 2 * c) * 32 + lane], h1 = u[(9 + 2 * c) * 32 + lane];
    const uint32_t ql[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                             l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
    const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int is = 0; is < 2; is++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        // elements 128c + 32i + 16is .. +15: limb words 32c + 8i + 4is .. +3
        const uint4 la = ((const uint4 *)xa)[8 * c + 2 * i + is];
        const uint4 lb = ((const uint4 *)xb)[8 * c + 2 * i + is];
        const uint4 lc = ((const uint4 *)xc)[8 * c + 2 * i + is];
        const uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
                       c4[4] = {lc.x, lc.y, lc.z, lc.w};
        int A = 0, B = 0, C = 0;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const int k = 4 * is + kk;
          const uint32_t L = i & 1 ? ql[8 + k] : ql[k];
          const uint32_t H = qh[k];
          uint32_t q;
          if (i == 0) q = (L & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
          else if (i == 1) q = (L & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
          else if (i == 2) q = ((L >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
          else q = ((L >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
          A = gb_dp4a_us(q, a4[kk], A);
          B = gb_dp4a_us(q, b4[kk], B);
          C = gb_dp4a_us(q, c4[kk], C);
        }
        const float S = (float)A + (float)(254 * B + C) * kL2;
        const int si = 8 * c + is + 2 * i;  // scale of this 16-element sub-block
        const float sc = (float)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xFFu);
        acc = fmaf(sc, fmaf(xs[4 * c + i], S, -32.f * xsum[8 * c + 2 * i + is]), acc);
      }
    }
  }
  return d * acc;
}

// Q4_0: eight 32-element blocks per super-block, y = d*(q-8).
template <>
GB_DEV float sb_dot<GB_T_Q4_0>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  const uint4 h = u[lane];
  const uint32_t dw[4] = {h.x, h.y, h.z, h.w};
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint4 q = u[(1 + k) * 32 + lane];
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const uint4 la = ((const uint4 *)xa)[2 * k], ha = ((const uint4 *)xa)[2 * k + 1];
    const uint4 lb = ((const uint4 *)xb)[2 * k], hb = ((const uint4 *)xb)[2 * k + 1];
    const uint4 lc = ((const uint4 *)xc)[2 * k], hc = ((const uint4 *)xc)[2 * k + 1];
    const uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
                   c4[4] = {lc.x, lc.y, lc.z, lc.w};
    const uint32_t A4[4] = {ha.x, ha.y, ha.z, ha.w}, B4[4] = {hb.x, hb.y, hb.z, hb.w},
                   C4[4] = {hc.x, hc.y, hc.z, hc.w};
    int Al = 0, Bl = 0, Cl = 0, Ah = 0, Bh = 0, Ch = 0;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint32_t lo = qw[kk] & 0x0F0F0F0Fu, hi = qw[kk] & 0xF0F0F0F0u;
      Al = gb_dp4a_us(lo, a4[kk], Al);
      Bl = gb_dp4a_us(lo, b4[kk], Bl);
      Cl = gb_dp4a_us(lo, c4[kk], Cl);
      Ah = gb_dp4a_us(hi, A4[kk], Ah);
      Bh = gb_dp4a_us(hi, B4[kk], Bh);
      Ch = gb_dp4a_us(hi, C4[kk], Ch);
    }
    const int A = 16 * Al + Ah, B = 16 * Bl + Bh, C = 16 * Cl + Ch;
    const float S = ((float)A + (float)(254 * B + C) * kL2) * 0.0625f;
    const float dk = gb_half_to_float((uint16_t)((dw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu));
    acc = fmaf(dk, fmaf(xs[k], S, -8.f * (xsum[2 * k] + xsum[2 * k + 1])), acc);
  }
  return acc;
}

// ---- epilogues (one warp, lane l = row 32*rowblock + l) ---------------------

GB_DEV uint64_t argmax_key(float v, uint32_t idx) {
  // larger value wins, then the lower index (model.Argmax, model/model.go:376)
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

struct Kp {  // kernel parameters
  GbGemvArgs a;
  int rb, nrb;
  int K;            // units per ring stage
  int nstage;       // ring stages (at most kMaxStages)
  int stage_bytes;  // bytes of one stage buffer (K units of the larger type)
  int xs_max;       // super-blocks of activation staged per CTA
  unsigned units;
};

constexpr int kMaxStages = 8;

template <int EPI>
GB_DEV void epilogue(const Kp &p, int rbk, float y0, float y1) {
  const GbGemvArgs &a = p.a;
  const GbEpiArgs &e = a.e;
  const int lane = threadIdx.x & 31;
  if constexpr (EPI == GB_EPI_PLAIN) {
    int r = rbk * 32 + lane;
    if (r < a.rows) e.y[r] = y0;
  } else if constexpr (EPI == GB_EPI_RESID) {
    int r = rbk * 32 + lane;
    float xn = e.x[r] + y0;  // cpu.Add, backend/cpu/cpu.go:60
    e.x[r] = xn;
    GbXPack pk{e.out_pack.a, e.out_pack.b, e.out_pack.c, e.out_pack.s, e.out_pack.sum16, e.out_pack.ssq};
    gb_pack_group(pk, rbk, xn * e.wnorm[r]);
    float ss = gb_warp_sum(xn * xn);
    if (lane == 0) pk.ssq[rbk] = ss;
  } else if constexpr (EPI == GB_EPI_SWIGLU) {  // cpu.SiluMul, backend/cpu/cpu.go:53
    float g = y0, u = y1;
    float ex = (float)exp(-(double)g);
    float act = g / (1.f + ex) * u;
    GbXPack pk{e.out_pack.a, e.out_pack.b, e.out_pack.c, e.out_pack.s, e.out_pack.sum16, nullptr};
    gb_pack_group(pk, rbk, act);
  } else if constexpr (EPI == GB_EPI_QKV) {
    int r = rbk * 32 + lane;
    int pos = *e.pos;
    bool ok = pos >= 0 && pos < e.max_len;
    if (!ok) {
      if (lane == 0 && e.err) atomicOr(e.err, GB_DEVERR_POS);
      return;
    }
    const int hd = e.head_dim;
    float partner = __shfl_xor_sync(0xffffffffu, y0, 1);
    float out = y0;
    if (r < e.q_rows + e.kv_rows) {  // cpu.RoPE, backend/cpu/cpu.go:69 (float64 math)
      int rr = r < e.q_rows ? r : r - e.q_rows;
      int j = (rr % hd) >> 1;
      const double *cs = e.rope_cs + ((size_t)pos * (hd / 2) + j) * 2;
      double c = cs[0], s = cs[1];
      double x0 = (lane & 1) ? (double)partner : (double)y0;
      double x1 = (lane & 1) ? (double)y0 : (double)partner;
      out = (lane & 1) ? (float)__dadd_rn(__dmul_rn(x0, s), __dmul_rn(x1, c))
                       : (float)__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, s));
    }
    if (r < e.q_rows) {
      e.q_out[r] = out;
    } else if (r < e.q_rows + e.kv_rows) {
      int rr = r - e.q_rows, h = rr / hd, dd = rr % hd;
      if (e.kv_f16) {
        size_t idx = (((size_t)h * (hd / 8) + dd / 8) * e.max_len + pos) * 8 + (dd & 7);
        ((uint16_t *)e.kcache)[idx] = gb_float_to_half_rn(out);
      } else {
        size_t idx = (((size_t)h * (hd / 4) + dd / 4) * e.max_len + pos) * 4 + (dd & 3);
        ((float *)e.kcache)[idx] = out;
      }
    } else if (r < e.q_rows + 2 * e.kv_rows) {
      int rr = r - e.q_rows - e.kv_rows, h = rr / hd, dd = rr % hd;
      if (e.kv_f16) {  // fp16 V: the K layout
        size_t idx = (((size_t)h * (hd / 8) + dd / 8) * e.max_len + pos) * 8 + (dd & 7);
        ((uint16_t *)e.vcache)[idx] = gb_float_to_half_rn(out);
      } else {
        ((float *)e.vcache)[((size_t)h * e.max_len + pos) * hd + dd] = out;
      }
    }
  } else if constexpr (EPI == GB_EPI_LOGITS) {
    int r = rbk * 32 + lane;
    uint32_t gidx = (uint32_t)(e.row_offset + r);
    uint64_t key = 0;
    if (r < a.rows) {
      e.y[r] = y0;
      float v = y0;
      // NaN never wins, except at index 0 where model.Argmax keeps it.
      if (isnan(v)) v = gidx == 0 ? INFINITY : -INFINITY;
      key = argmax_key(v, gidx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      uint64_t k2 = __shfl_xor_sync(0xffffffffu, key, o);
      key = k2 > key ? k2 : key;
    }
    if (lane == 0) {
      atomicMax(e.best, (unsigned long long)key);
      __threadfence();
      unsigned done = atomicAdd(e.counter, 1u);
      if (done + 1 == (unsigned)p.nrb) {
        __threadfence();
        unsigned long long k = atomicAdd(e.best, 0ull);
        int32_t tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        if (e.token_out) *e.token_out = tok;
        if (e.key_out) *e.key_out = k;  // tensor parallel: reduced across ranks next
        if (e.token_hist) {
          int pos = *e.pos;
          if (pos >= 0 && pos < e.max_len) e.token_hist[pos] = tok;
        }
        *e.best = 0ull;
        *e.counter = 0u;
      }
    }
  }
}

// CTA b of G owns units [U*b/G, U*(b+1)/G) (the product fits 64 bits).
GB_DEV unsigned ubeg(unsigned U, unsigned G, unsigned b) {
  return (unsigned)(((unsigned long long)U * b) / G);
}
// CTA whose range contains unit u.
GB_DEV unsigned cta_of_unit(unsigned U, unsigned G, unsigned u) {
  unsigned b = (unsigned)(((unsigned long long)u * G) / U);
  while (b > 0 && ubeg(U, G, b) > u) b--;
  while (b + 1 < G && ubeg(U, G, b + 1) <= u) b++;
  return b;
}

template <int T>
__device__ __noinline__ float sb_dot_outlined(const uint8_t *st, int lane, const uint32_t *xa,
                                              const uint32_t *xb, const uint32_t *xc, const float *xs,
                                              const float *xsum) {
  return sb_dot<T>(st, lane, xa, xb, xc, xs, xsum);
}

template <int TA, int TB>
GB_DEV float decode(int ty, const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xs, const float *xsum) {
  if (TA == TB || ty == TA) return sb_dot<TA>(st, lane, xa, xb, xc, xs, xsum);
  return sb_dot<TB>(st, lane, xa, xb, xc, xs, xsum);
}

// Byte offset of unit u (row-block u / nsb, super-block u % nsb) in the tiled
// weights. Units are contiguous in this order: 32-row tiles are tile-major
// and super-block-minor, the type-B tiles follow the type-A ones, and a
// gate/up row-block holds the gate and up sb-blocks of each super-block side
// by side. So any run of units is one contiguous byte range.
template <int TA, int TB>
GB_DEV size_t unit_off(const Kp &p, unsigned u) {
  const size_t ua = (size_t)p.rb * gb_tiled_sb_bytes(TA);
  if (TA == TB) return (size_t)u * ua;
  const unsigned split_u = (unsigned)p.a.split_tile * (unsigned)p.a.nsb;  // rb is 1 here
  return u < split_u ? (size_t)u * ua : (size_t)split_u * ua + (size_t)(u - split_u) * gb_tiled_sb_bytes(TB);
}

// Named barrier over the W consumer warps (the producer warp never joins).
template <int W>
GB_DEV void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(W * 32) : "memory"); }

// One CTA owns the contiguous unit range [cu0, cu1) (stream-K over the
// persistent grid, or one row-block per CTA). A producer warp streams the
// range through a ring of shared-memory stages, each stage K consecutive
// units moved by ONE 1-D TMA bulk copy (tens of KB: few copies and few
// mbarrier phases keep the copy engine at HBM speed). Consumer warps take
// the units round-robin (unit j of the CTA goes to warp j mod W), decode them
// against the activation pack and release each unit's slot through the
// stage's `empty` mbarrier, which completes after K releases. The CTA's
// range is cut into segments, one per row-block it touches; at a segment's
// end the warps' partial sums are added in warp order by one reducer warp
// (deterministic), and only a segment that continues in another CTA goes
// through global memory.
template <int TA, int TB, int EPI, int W>
__global__ void __launch_bounds__(32 * (W + 1), W <= 8 ? 2 : 1) gemv_kernel(const Kp p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GbGemvArgs &a = p.a;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nsb = a.nsb, K = p.K, NS = p.nstage;
  const unsigned U = p.units, G = gridDim.x, b = blockIdx.x;
  const unsigned cu0 = ubeg(U, G, b), cu1 = ubeg(U, G, b + 1);
  const unsigned nst = (cu1 - cu0 + (unsigned)K - 1) / (unsigned)K;  // stages of this CTA

  // shared memory: [NS] stages | pack planes a,b,c | scales | sums | 2 x [W][64] segment partials
  uint8_t *ring = smem;
  const int XS = p.xs_max;
  uint8_t *xbase = smem + (size_t)NS * p.stage_bytes;
  uint32_t *xa_s = (uint32_t *)xbase;
  uint32_t *xb_s = xa_s + XS * 64;
  uint32_t *xc_s = xb_s + XS * 64;
  float *xs_s = (float *)(xc_s + XS * 64);
  float *xsum_s = xs_s + XS * 8;
  float *psum = xsum_s + XS * 16;  // [2][W][64]
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ double red[W];
  __shared__ float inv_s;

  // 0. let the next kernel's CTAs start (they stream their weights meanwhile)
  gb_grid_dep_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      gb_mbar_init(&full[s], 1);
      gb_mbar_init(&empty[s], (uint32_t)K);
    }
    gb_mbar_fence_init();
  }
  __syncthreads();

  if (warp == W) {
    // 1. producer: weights do not depend on the previous kernel
    if (lane == 0) {
      unsigned k = 0;
      for (; k < nst; k++) {
        const int s = (int)(k % (unsigned)NS);
        if (k >= (unsigned)NS) {
          if (!gb_mbar_wait(&empty[s], (k / NS - 1) & 1)) {
            if (a.e.err) atomicOr(a.e.err, GB_DEVERR_TIMEOUT);
            break;
          }
          gb_fence_proxy_async();
        }
        const unsigned j0 = cu0 + k * (unsigned)K, j1 = min(cu1, j0 + (unsigned)K);
        const size_t o0 = unit_off<TA, TB>(p, j0), o1 = unit_off<TA, TB>(p, j1);
        gb_mbar_expect_tx(&full[s], (uint32_t)(o1 - o0));
        gb_bulk_g2s(ring + (size_t)s * p.stage_bytes, a.w + o0, (uint32_t)(o1 - o0), &full[s]);
      }
      // the copies still in flight land (bounded) before the CTA exits
      for (unsigned j = k > (unsigned)NS ? k - NS : 0; j < k; j++)
        (void)gb_mbar_wait(&full[j % NS], (j / NS) & 1);
    }
    return;
  }

  // 2. the activation pack (and the norm's sums of squares) come from the
  // preceding kernel: one round trip for all of it
  constexpr int CT = W * 32;
  const int tid = threadIdx.x;
  gb_grid_dep_wait();
  const int nsbs = (cu1 - cu0) >= (unsigned)nsb ? nsb : (int)(cu1 - cu0);
  const int sbf = (int)(cu0 % (unsigned)nsb);
  {
    double ss = 0;
    if (a.in_ssq)
      for (int g = tid; g < nsb * 8; g += CT) ss += (double)__ldcg(a.in_ssq + g);
    for (int i = tid; i < nsbs * 48; i += CT) {  // 3 planes x 16 uint4 per sb
      const int plane = i / (nsbs * 16), rest = i - plane * (nsbs * 16);
      const int ls = rest >> 4, v = rest & 15;
      int sb = sbf + ls;
      if (sb >= nsb) sb -= nsb;
      const int8_t *src = plane == 0 ? a.in.a : plane == 1 ? a.in.b : a.in.c;
      uint32_t *dst = plane == 0 ? xa_s : plane == 1 ? xb_s : xc_s;
      ((uint4 *)(dst + ls * 64))[v] = __ldcg((const uint4 *)(src + sb * 256) + v);
    }
    for (int i = tid; i < nsbs * 24; i += CT) {
      const int ls = i / 24, v = i - ls * 24;
      int sb = sbf + ls;
      if (sb >= nsb) sb -= nsb;
      if (v < 8)
        xs_s[ls * 8 + v] = __ldcg(a.in.s + sb * 8 + v);
      else
        xsum_s[ls * 16 + v - 8] = __ldcg(a.in.sum16 + sb * 16 + v - 8);
    }
    if (a.in_ssq) {  // cpu.RMSNorm, backend/cpu/cpu.go:17: inv = 1/sqrt(sum/n + eps), float64
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red[warp] = ss;
      consumers_sync<W>();
      if (tid == 0) {
        double t = 0;
        for (int w2 = 0; w2 < W; w2++) t += red[w2];
        inv_s = (float)(1.0 / sqrt(t / (double)(nsb * 256) + (double)a.eps));
      }
      consumers_sync<W>();
      const float inv = inv_s;
      for (int i = tid; i < nsbs * 24; i += CT) {
        const int ls = i / 24, v = i - ls * 24;
        if (v < 8) xs_s[ls * 8 + v] *= inv;
        else xsum_s[ls * 16 + v - 8] *= inv;
      }
    }
  }
  consumers_sync<W>();

  // 3. units round-robin over the warps, segment by segment
  const size_t sbb_a = (size_t)gb_tiled_sb_bytes(TA);
  bool timeout = false;
  unsigned j = (unsigned)warp;  // this warp's next unit (CTA-relative)
  int nseg = 0;
  for (unsigned s0 = cu0; s0 < cu1; nseg++) {
    const int rbk = (int)(s0 / (unsigned)nsb);
    const unsigned s1 = min(cu1, (unsigned)(rbk + 1) * (unsigned)nsb);
    float acc0 = 0.f, acc1 = 0.f;
    for (; cu0 + j < s1; j += W) {
      const unsigned u = cu0 + j, k = j / (unsigned)K;
      const int s = (int)(k % (unsigned)NS);
      if (!timeout && !gb_mbar_wait(&full[s], (k / NS) & 1)) timeout = true;
      if (!timeout) {
        int ls = (int)(u % (unsigned)nsb) - sbf;
        if (ls < 0) ls += nsb;
        const uint32_t *xa = xa_s + ls * 64, *xb = xb_s + ls * 64, *xc = xc_s + ls * 64;
        const float *xs = xs_s + ls * 8, *xsum = xsum_s + ls * 16;
        const uint8_t *st = ring + (size_t)s * p.stage_bytes +
                            (unit_off<TA, TB>(p, u) - unit_off<TA, TB>(p, cu0 + k * (unsigned)K));
        if constexpr (EPI == GB_EPI_SWIGLU) {
          // gate then up sb-block; one decode at a time keeps the register
          // footprint of a single tile
          acc0 += sb_dot_outlined<TA>(st, lane, xa, xb, xc, xs, xsum);
          acc1 += sb_dot_outlined<TA>(st + sbb_a, lane, xa, xb, xc, xs, xsum);
        } else {
          acc0 += decode<TA, TB>(rbk < a.split_tile ? TA : TB, st, lane, xa, xb, xc, xs, xsum);
        }
      }
      __syncwarp();
      if (lane == 0) gb_mbar_arrive(&empty[s]);
    }
    float *ps = psum + (size_t)(nseg & 1) * W * 64;
    ps[warp * 64 + lane] = acc0;
    ps[warp * 64 + 32 + lane] = acc1;
    consumers_sync<W>();
    if (warp == nseg % W) {  // reducer of this segment (sum in warp order)
      float y0 = 0.f, y1 = 0.f;
      for (int w2 = 0; w2 < W; w2++) {
        y0 += ps[w2 * 64 + lane];
        y1 += ps[w2 * 64 + 32 + lane];
      }
      const unsigned R0 = (unsigned)rbk * nsb, R1 = R0 + nsb;
      if (s0 == R0 && s1 == R1) {
        epilogue<EPI>(p, rbk, y0, y1);
      } else {
        // the row-block continues in another CTA: global partial per CTA
        const int which = cu0 >= R0 ? 0 : 1;
        float *slot = a.e.part + ((size_t)b * 2 + which) * 64;
        slot[lane] = y0;
        slot[32 + lane] = y1;
        __threadfence();
        __syncwarp();
        unsigned done = 0;
        if (lane == 0) done = atomicAdd(a.e.tile_counter + rbk, s1 - s0) + (s1 - s0);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done == (unsigned)nsb) {
          __threadfence();
          const unsigned bf = cta_of_unit(U, G, R0), bl = cta_of_unit(U, G, R1 - 1);
          float z0 = 0.f, z1 = 0.f;
          for (unsigned b2 = bf; b2 <= bl; b2++) {
            const unsigned c0 = ubeg(U, G, b2), c1 = ubeg(U, G, b2 + 1);
            if (c0 == c1) continue;
            const float *sl = a.e.part + ((size_t)b2 * 2 + (c0 >= R0 ? 0 : 1)) * 64;
            z0 += __ldcg(sl + lane);
            z1 += __ldcg(sl + 32 + lane);
          }
          if (lane == 0) a.e.tile_counter[rbk] = 0u;
          epilogue<EPI>(p, rbk, z0, z1);
        }
      }
    }
    s0 = s1;
  }
  if (timeout && lane == 0 && a.e.err) atomicOr(a.e.err, GB_DEVERR_TIMEOUT);
}

// ---- repack raw ggml rows into the tiled layout (load time) ---------------
__global__ void repack_kernel(int typ, const uint8_t *raw, int rows, int nsb, int ntiles,
                              uint8_t *out) {
  const long long sbb = gb_tiled_sb_bytes(typ);
  const long long rawsb = gb_sb_raw_bytes(typ);
  const long long rowbytes = rawsb * nsb;
  const long long total = (long long)ntiles * nsb * 32;  // (tile, sb, lane)
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int lane = (int)(i % 32);
    long long ts = i / 32;
    int sb = (int)(ts % nsb), tile = (int)(ts / nsb);
    int row = tile * 32 + lane;
    uint8_t *dst = out + ((long long)tile * nsb + sb) * sbb;
    const uint8_t *src = raw + (long long)row * rowbytes + (long long)sb * rawsb;
    for (int b = 0; b < rawsb; b++) dst[gb_tiled_offset(typ, lane, b)] = row < rows ? src[b] : 0;
  }
}

// ---- standalone limb pack of a float vector (one warp per group) ---------
__global__ void pack_kernel(const float *x, int n, GbXPackBuf p) {
  int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (g >= n / 32) return;
  GbXPack pk{p.a, p.b, p.c, p.s, p.sum16, nullptr};
  gb_pack_group(pk, g, x[g * 32 + (threadIdx.x & 31)]);
}

int g_sms = 0;
int sms() {
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  return g_sms;
}

size_t gemv_smem(int warps, int nstage, int stage_bytes, int xs_max) {
  return (size_t)nstage * stage_bytes + (size_t)xs_max * (3 * 256 + 4 * 24) + (size_t)2 * warps * 64 * 4;
}

using KernelFn = void (*)(Kp);

template <int TA, int TB, int W>
KernelFn pick_epi(int epi) {
  switch (epi) {
    case GB_EPI_PLAIN: return gemv_kernel<TA, TB, GB_EPI_PLAIN, W>;
    case GB_EPI_QKV: return gemv_kernel<TA, TB, GB_EPI_QKV, W>;
    case GB_EPI_RESID: return gemv_kernel<TA, TB, GB_EPI_RESID, W>;
    case GB_EPI_SWIGLU: return gemv_kernel<TA, TB, GB_EPI_SWIGLU, W>;
    case GB_EPI_LOGITS: return gemv_kernel<TA, TB, GB_EPI_LOGITS, W>;
  }
  return nullptr;
}

template <int W>
KernelFn pick_w(int ta, int tb, int epi) {
  if (ta == tb) {
    if (ta == GB_T_Q4_K) return pick_epi<GB_T_Q4_K, GB_T_Q4_K, W>(epi);
    if (ta == GB_T_Q6_K) return pick_epi<GB_T_Q6_K, GB_T_Q6_K, W>(epi);
    if (ta == GB_T_Q4_0) return pick_epi<GB_T_Q4_0, GB_T_Q4_0, W>(epi);
  } else if (ta == GB_T_Q4_K && tb == GB_T_Q6_K && epi == GB_EPI_QKV) {
    return gemv_kernel<GB_T_Q4_K, GB_T_Q6_K, GB_EPI_QKV, W>;
  } else if (ta == GB_T_Q6_K && tb == GB_T_Q4_K && epi == GB_EPI_QKV) {
    return gemv_kernel<GB_T_Q6_K, GB_T_Q4_K, GB_EPI_QKV, W>;
  }
  return nullptr;
}

KernelFn pick(int ta, int tb, int epi, int warps) {
  return warps == 16 ? pick_w<16>(ta, tb, epi) : pick_w<8>(ta, tb, epi);
}

int smem_optin() {
  static int v = 0;
  if (!v) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (v <= 0) v = 227 * 1024;
  }
  return v;
}

}  // namespace

size_t gb_tiled_bytes(int typ, int rows, int cols) {
  int ntiles = (rows + 31) / 32;
  return (size_t)ntiles * (cols / 256) * gb_tiled_sb_bytes(typ);
}

int gb_repack_launch(int typ, const uint8_t *raw, int rows, int cols, uint8_t *tiled,
                     cudaStream_t st) {
  if (!gb_tiled_type(typ) || cols % 256)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: repack: %d columns of type %d", cols, typ);
  int ntiles = (rows + 31) / 32, nsb = cols / 256;
  long long total = (long long)ntiles * nsb * 32;
  long long blocks = (total + 255) / 256;
  if (blocks > 65535LL * 8) blocks = 65535LL * 8;
  repack_kernel<<<(unsigned)blocks, 256, 0, st>>>(typ, raw, rows, nsb, ntiles, tiled);
  GB_CUDA(cudaGetLastError(), "gpu: repack");
  return GB_OK;
}

int gb_pack_launch(const float *x, int n, const GbXPackBuf &p, cudaStream_t st) {
  if (n % 32) return gb_fail(GB_ERR_INVALID, "gpu: pack: %d is not a multiple of 32", n);
  int groups = n / 32;
  pack_kernel<<<(groups + 7) / 8, 256, 0, st>>>(x, n, p);
  GB_CUDA(cudaGetLastError(), "gpu: pack");
  return GB_OK;
}

GbGemvPlan gb_gemv_plan(int ntiles, int nsb, int epi, int nsm) {
  GbGemvPlan p;
  p.rb = epi == GB_EPI_SWIGLU ? 2 : 1;
  p.warps = 8;
  p.stages = 2;
  p.ks = 1;
  (void)ntiles;
  (void)nsb;
  (void)nsm;
  return p;
}

int gb_gemv_scratch_floats(int ntiles, const GbGemvPlan &p) {
  (void)ntiles;
  (void)p;
  // two 64-float partial slots per warp of the persistent grid (<= 8 CTAs of 8 warps per SM)
  return sms() * 8 * 8 * 2 * 64;
}

int gb_gemv_launch(const GbGemvArgs &a, const GbGemvPlan &plan, cudaStream_t st, bool pdl) {
  if (a.nsb <= 0 || a.ntiles <= 0) return gb_fail(GB_ERR_INVALID, "gpu: gemv: empty matrix");
  Kp p;
  p.a = a;
  p.rb = plan.rb;
  if (a.ntiles % p.rb) return gb_fail(GB_ERR_INVALID, "gpu: gemv: tiles not paired");
  const int ta = a.type_a, tb = a.split_tile < a.ntiles ? a.type_b : a.type_a;
  p.a.type_b = tb;
  // consumer warps per CTA: 16 (a whole SM) or 8 (half an SM); GB_GEMV_WARPS overrides
  int warps = 16;
  if (const char *e = getenv("GB_GEMV_WARPS")) warps = atoi(e) == 8 ? 8 : 16;
  KernelFn fn = pick(ta, tb, a.epi, warps);
  if (!fn) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: types %d/%d with epilogue %d", ta, tb, a.epi);
  if (p.rb == 2 && ta != tb) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: gate/up types differ");
  p.nrb = a.ntiles / p.rb;
  p.units = (unsigned)p.nrb * (unsigned)a.nsb;
  const int ub = p.rb * std::max(gb_tiled_sb_bytes(ta), gb_tiled_sb_bytes(tb));  // largest unit
  const int nsm = sms();
  const long long cap = smem_optin();
  // opt in to the shared memory and learn the register count (once per kernel)
  static KernelFn seen[64];
  static int seen_static[64];
  static int nseen = 0;
  int static_smem = -1;
  for (int i = 0; i < nseen; i++)
    if (seen[i] == fn) static_smem = seen_static[i];
  if (static_smem < 0) {
    cudaFuncAttributes fa;
    GB_CUDA(cudaFuncGetAttributes(&fa, fn), "gpu: gemv");
    static_smem = (int)fa.sharedSizeBytes;
    GB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(cap - static_smem)),
            "gpu: gemv: shared memory attribute");
    if (nseen < 64) {
      seen[nseen] = fn;
      seen_static[nseen++] = static_smem;
    }
  }
  // Launch shape. Grid: one row-block per CTA when there are at most as many
  // row-blocks as SMs (no partial sums leave the CTA), else one persistent CTA
  // per SM over a contiguous range of units. Either way a CTA uses about half
  // an SM (GB_SMEM_BUDGET bytes of shared memory, 288 threads of at most 112
  // registers), so the next kernel's CTA fits beside it and starts streaming
  // its own weights during this kernel's tail. Ring: stages of K units of
  // about 36 KB, as many stages as the budget holds (2 to 8).
  // GB_GEMV_RING_<PLAIN|QKV|RESID|SWIGLU|LOGITS> or GB_GEMV_RING = "K,stages"
  // force the ring (sweeps) when it fits.
  static const char *epi_names[] = {"PLAIN", "QKV", "RESID", "SWIGLU", "LOGITS"};
  int fk = 0, fs = 0;
  {
    char key[64];
    snprintf(key, sizeof key, "GB_GEMV_RING_%s", epi_names[a.epi]);
    const char *e = getenv(key);
    if (!e) e = getenv("GB_GEMV_RING");
    if (e && sscanf(e, "%d,%d", &fk, &fs) != 2) fk = fs = 0;
  }
  long long grid = p.nrb <= nsm ? p.nrb : std::min<long long>(nsm, p.units);
  if (grid * 128 > (long long)gb_gemv_scratch_floats(a.ntiles, plan)) grid = gb_gemv_scratch_floats(a.ntiles, plan) / 128;
  const int upc = (int)((p.units + grid - 1) / grid);  // units per CTA (at most)
  const int xs = std::min(a.nsb, upc + 1);
  long long budget = warps == 8 ? 113 * 1024 : 220 * 1024;
  if (const char *e = getenv("GB_SMEM_BUDGET")) budget = atoll(e);
  const long long room = cap - static_smem;
  const long long fixed = (long long)gemv_smem(warps, 0, 0, xs);
  int K = std::max(1, std::min(16, (36 * 1024 + ub / 2) / ub)), ns = 0;
  K = std::min(K, upc);
  if (fk > 0 && fs >= 2 && fs <= kMaxStages && fixed + (long long)fs * fk * ub <= room) {
    K = fk;
    ns = fs;
  } else {
    for (;; K--) {
      ns = (int)std::min<long long>(kMaxStages, (budget - fixed) / ((long long)K * ub));
      if (ns >= 2 || K == 1) break;
    }
    if (ns < 2) ns = 2;
  }
  p.K = K;
  p.nstage = ns;
  p.stage_bytes = (K * ub + 127) / 128 * 128;
  p.xs_max = xs;
  const size_t smem = gemv_smem(warps, ns, p.stage_bytes, xs);
  if ((long long)smem > room)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: %zu B of shared memory for %d stages of %d units", smem, ns, K);
  if (getenv("GB_GEMV_VERBOSE"))
    fprintf(stderr, "gemv epi=%s types=%d/%d units=%u rb=%d: grid=%lld warps=%d K=%d stages=%d stage=%d smem=%zu forced=%d,%d\n",
            epi_names[a.epi], ta, tb, p.units, p.rb, grid, warps, K, ns, p.stage_bytes, smem, fk, fs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)(32 * (warps + 1)));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t le = cudaLaunchKernelEx(&cfg, fn, p);
  if (le != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, fn);
    return gb_fail(GB_ERR_CUDA, "gpu: gemv launch: %s (grid %lld, %d stages of %d units, %zu B shared, max %d B, static %zu B)",
                   cudaGetErrorString(le), grid, ns, K, smem, fa.maxDynamicSharedSizeBytes,
                   (size_t)fa.sharedSizeBytes);
  }
  return GB_OK;
}
