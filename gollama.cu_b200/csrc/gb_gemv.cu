// gb_gemv.cu -- batch-1 quantized matrix-vector products on the tiled layout
// (gb_formats.h), with fused epilogues for the decode step.
//
// Replaces kernels.MatVecQ4_0 / MatVecQ4K / MatVecQ6K (kernels/quantmv.go:18-136)
// on the model path. Design:
//  * Work is the list of units: sb-blocks (32 rows x 256 columns) in
//    (row-block, super-block) order. A row-block is one 32-row tile, or for
//    the SwiGLU epilogue a gate/up tile pair whose gate and up sb-blocks are
//    two units. Every CTA takes one contiguous range of units (stream-K over
//    a persistent grid, or one row-block per CTA for small matrices), so all
//    SMs stay busy whatever the matrix shape and no wave is partial.
//  * Units are contiguous in memory in that order, so a CTA's range is one
//    byte range. A producer warp streams it through a ring of shared-memory
//    stages of K units (tens of KB) with one 1-D TMA bulk copy per stage;
//    16 consumer warps decode the units round-robin and give each stage back
//    through an mbarrier. Lane l of a warp owns row l of the tile; with an
//    even warp count a warp sees only gate or only up units of a pair.
//  * The activation is staged per CTA as three int8 limbs per element with
//    one scale per 256-element super-block (RMSNorm applied first when the
//    GEMV consumes a normalised input), so the 4-bit / 6-bit quants meet it
//    in dp4a (4 products per instruction, exact int32 sums) and the ggml
//    sub-block scales are applied in int32; float math once per super-block.
//  * A row-block split between CTAs is finished by the CTA whose atomic
//    count completes it; it sums the partials in CTA order (deterministic)
//    and runs the epilogue. Counters are reset by that CTA, so the kernel can
//    be replayed from a CUDA graph.
//  * Under programmatic dependent launch the next kernel is launched at this
//    kernel's start; its producer streams its own weights as soon as its CTAs
//    find room.
//  * One instantiation per (weight types, epilogue) keeps each kernel's code
//    small.
#include <math.h>
#include <stdlib.h>

#include <algorithm>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr float kL2 = 1.f / 64516.f;  // 1/254^2: limbs b, c are combined as 254*b + c


// ---- per-super-block decode + dot products. `st` is the sb-block in shared
// memory; xa/xb/xc are the limb planes (as 32-bit words) of the block's 256
// activation elements (one scale xs for all 256: x ~ xs*(a + b/254 + c/254^2)),
// xsum the 16 sums of 16 activation values and sl the 16 per-16 limb sums
// (int16 a, b, c sums packed in a uint2). The integer dot products of every
// sub-block are weighted by its integer scale in int32 and converted to float
// once per super-block.
template <int T>
GB_DEV float sb_dot(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xsum, const uint2 *sl, float xs);

GB_DEV int lo16(uint32_t w) { return (int)(int16_t)(w & 0xFFFFu); }
GB_DEV int hi16(uint32_t w) { return (int)(int16_t)(w >> 16); }
GB_DEV int byte_i(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); }

// Q4_K: quant/quant.go:97 layout; kernels/quantmv.go:66 factorisation
// sum = d*sum_j sc_j*(q.x)_j - dmin*sum_j m_j*(sum x)_j. The high nibbles are
// used in place (16*q), so their family of sums carries a factor 16.
template <>
GB_DEV float sb_dot<GB_T_Q4_K>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  (void)sl;
  const uint4 *u = (const uint4 *)st;
  const uint4 h = u[lane];
  const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFFu));
  const float dmin = gb_half_to_float((uint16_t)(h.x >> 16));
  const uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
  const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  int IA0 = 0, IB0 = 0, IC0 = 0, IA1 = 0, IB1 = 0, IC1 = 0;
  float tm = 0.f;
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
    const int j0 = 2 * c, j1 = 2 * c + 1;
    const int sc0 = byte_i(j0 < 4 ? sc03 : sc47, j0 & 3), sc1 = byte_i(j1 < 4 ? sc03 : sc47, j1 & 3);
    IA0 += sc0 * A0;
    IB0 += sc0 * B0;
    IC0 += sc0 * C0;
    IA1 += sc1 * A1;
    IB1 += sc1 * B1;
    IC1 += sc1 * C1;
    const float m0 = (float)byte_i(j0 < 4 ? m03 : m47, j0 & 3), m1 = (float)byte_i(j1 < 4 ? m03 : m47, j1 & 3);
    tm = fmaf(m0, xsum[4 * c] + xsum[4 * c + 1], tm);
    tm = fmaf(m1, xsum[4 * c + 2] + xsum[4 * c + 3], tm);
  }
  // sum sc*q*x / xs = A + (254 B + C)/254^2 per family; |I| < 2^28, float error 2^-24
  const float A = (float)IA0 + (float)IA1 * 0.0625f, B = (float)IB0 + (float)IB1 * 0.0625f,
              C = (float)IC0 + (float)IC1 * 0.0625f;
  return d * (xs * (A + (254.f * B + C) * kL2)) - dmin * tm;
}

// Q5_K (ggml block_q5_K; the reference has no decoder for it): the Q4_K
// factorisation with 5-bit quants q = nibble | fifth bit << 4 (0..31). Both
// families are formed shifted (no factor 16: 16*31 does not fit a byte).
template <>
GB_DEV float sb_dot<GB_T_Q5_K>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  (void)sl;
  const uint4 *u = (const uint4 *)st;
  const uint4 h = u[lane];
  const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFFu));
  const float dmin = gb_half_to_float((uint16_t)(h.x >> 16));
  const uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
  const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  const uint4 qh0 = u[1 * 32 + lane], qh1 = u[2 * 32 + lane];
  const uint32_t qhw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
  int IA = 0, IB = 0, IC = 0;
  float tm = 0.f;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint4 q0 = u[(3 + 2 * c) * 32 + lane], q1 = u[(4 + 2 * c) * 32 + lane];
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
        const uint32_t w = qw[4 * v + k], hb5 = qhw[4 * v + k];
        const uint32_t lo = (w & 0x0F0F0F0Fu) | (((hb5 >> (2 * c)) & 0x01010101u) << 4);
        const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) | (((hb5 >> (2 * c + 1)) & 0x01010101u) << 4);
        A0 = gb_dp4a_us(lo, a4[k], A0);
        B0 = gb_dp4a_us(lo, b4[k], B0);
        C0 = gb_dp4a_us(lo, c4[k], C0);
        A1 = gb_dp4a_us(hi, A4[k], A1);
        B1 = gb_dp4a_us(hi, B4[k], B1);
        C1 = gb_dp4a_us(hi, C4[k], C1);
      }
    }
    const int j0 = 2 * c, j1 = 2 * c + 1;
    const int sc0 = byte_i(j0 < 4 ? sc03 : sc47, j0 & 3), sc1 = byte_i(j1 < 4 ? sc03 : sc47, j1 & 3);
    IA += sc0 * A0 + sc1 * A1;
    IB += sc0 * B0 + sc1 * B1;
    IC += sc0 * C0 + sc1 * C1;
    const float m0 = (float)byte_i(j0 < 4 ? m03 : m47, j0 & 3), m1 = (float)byte_i(j1 < 4 ? m03 : m47, j1 & 3);
    tm = fmaf(m0, xsum[4 * c] + xsum[4 * c + 1], tm);
    tm = fmaf(m1, xsum[4 * c + 2] + xsum[4 * c + 3], tm);
  }
  // |I| < 8 * 63 * 32 * 31 * 127 < 2^27: exact in int32, float error 2^-24
  return d * (xs * ((float)IA + (254.f * (float)IB + (float)IC) * kL2)) - dmin * tm;
}

// Q6_K: quant/quant.go:114 layout; y = d*sc*(q-32) over 16-element sub-blocks.
// The -32 enters the dp4a sums as their starting value -32*(limb sums).
template <>
GB_DEV float sb_dot<GB_T_Q6_K>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  (void)xsum;
  const uint4 *u = (const uint4 *)st;
  const uint4 scv = u[12 * 32 + lane];
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  const float d = gb_half_to_float(((const uint16_t *)(st + 13 * 512))[lane]);
  int IA = 0, IB = 0, IC = 0;
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
        // elements 128c + 32i + 16is .. +15: limb words 32c + 8i + 4is .. +3, 16-group g
        const int g = 8 * c + 2 * i + is;
        const uint4 la = ((const uint4 *)xa)[g];
        const uint4 lb = ((const uint4 *)xb)[g];
        const uint4 lc = ((const uint4 *)xc)[g];
        const uint2 o = sl[g];
        const uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
                       c4[4] = {lc.x, lc.y, lc.z, lc.w};
        int A = -32 * lo16(o.x), B = -32 * hi16(o.x), C = -32 * lo16(o.y);
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
        const int sc = (int)(int8_t)((scw[g >> 2] >> (8 * (g & 3))) & 0xFFu);  // scale of sub-block g
        IA += sc * A;
        IB += sc * B;
        IC += sc * C;
      }
    }
  }
  return d * (xs * ((float)IA + (254.f * (float)IB + (float)IC) * kL2));
}

// Q4_0: eight 32-element blocks per super-block, y = d*(q-8); the -8 enters
// the dp4a sums as their starting value (x16 for the high nibbles, used in place).
template <>
GB_DEV float sb_dot<GB_T_Q4_0>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  (void)xsum;
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
    const uint2 ol = sl[2 * k], oh = sl[2 * k + 1];
    const uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
                   c4[4] = {lc.x, lc.y, lc.z, lc.w};
    const uint32_t A4[4] = {ha.x, ha.y, ha.z, ha.w}, B4[4] = {hb.x, hb.y, hb.z, hb.w},
                   C4[4] = {hc.x, hc.y, hc.z, hc.w};
    int Al = -8 * lo16(ol.x), Bl = -8 * hi16(ol.x), Cl = -8 * lo16(ol.y);
    int Ah = -128 * lo16(oh.x), Bh = -128 * hi16(oh.x), Ch = -128 * lo16(oh.y);
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
    acc = fmaf(dk, S, acc);
  }
  return xs * acc;
}

// Q8_0: eight 32-element blocks per super-block, y = d*q with int8 q
// (quant/quant.go:44-55); signed x signed dp4a, one float FMA per block.
template <>
GB_DEV float sb_dot<GB_T_Q8_0>(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                               const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  (void)xsum;
  (void)sl;
  const uint4 *u = (const uint4 *)st;
  const uint4 h = u[lane];
  const uint32_t dw[4] = {h.x, h.y, h.z, h.w};
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint4 q0 = u[(1 + 2 * k) * 32 + lane], q1 = u[(2 + 2 * k) * 32 + lane];
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint4 la = ((const uint4 *)xa)[2 * k], ha = ((const uint4 *)xa)[2 * k + 1];
    const uint4 lb = ((const uint4 *)xb)[2 * k], hb = ((const uint4 *)xb)[2 * k + 1];
    const uint4 lc = ((const uint4 *)xc)[2 * k], hc = ((const uint4 *)xc)[2 * k + 1];
    const uint32_t a8[8] = {la.x, la.y, la.z, la.w, ha.x, ha.y, ha.z, ha.w};
    const uint32_t b8[8] = {lb.x, lb.y, lb.z, lb.w, hb.x, hb.y, hb.z, hb.w};
    const uint32_t c8[8] = {lc.x, lc.y, lc.z, lc.w, hc.x, hc.y, hc.z, hc.w};
    int A = 0, B = 0, C = 0;
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
      A = gb_dp4a_ss(qw[kk], a8[kk], A);
      B = gb_dp4a_ss(qw[kk], b8[kk], B);
      C = gb_dp4a_ss(qw[kk], c8[kk], C);
    }
    // |A|, |B|, |C| < 32*127*128; 254*B + C fits int32
    const float S = (float)A + (float)(254 * B + C) * kL2;
    const float dk = gb_half_to_float((uint16_t)((dw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu));
    acc = fmaf(dk, S, acc);
  }
  return xs * acc;
}

// ---- epilogues (one warp, lane l = row 32*rowblock + l) ---------------------

GB_DEV uint64_t argmax_key(float v, uint32_t idx) {
  // larger value wins, then the lower index (model.Argmax, model/model.go:376)
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

struct Kp;
using KernelFnF = void (*)(Kp);

struct Kp {  // kernel parameters
  GbGemvArgs a;
  int rb, nrb;      // rb: sb-blocks per unit (1); nrb: row-blocks
  int half;         // gate/up row-block pairs: unit u is the gate (u even) or up (u odd) sb-block
  int aux_w;        // 1: the norm weights of the staged super-blocks are copied to shared memory
  int aux_rope;     // doubles of the RoPE row copied to shared memory (QKV epilogue), else 0
  int upr;          // units per row-block (nsb, or 2*nsb for gate/up pairs)
  int lk;           // log2 of the units per ring stage (K = 1 << lk, K <= consumer warps)
  int nstage;       // ring stages (at most kMaxStages)
  int stage_bytes;  // bytes of one stage buffer (K units of the larger type)
  int xs_max;       // super-blocks of activation staged per CTA
  unsigned units;
};

constexpr int kMaxStages = 8;
constexpr int kPend = 4;  // segments reduced per barrier

template <int EPI>
GB_DEV void epilogue(const Kp &p, int rbk, float y0, float y1, const double *rope_row) {
  const GbGemvArgs &a = p.a;
  const GbEpiArgs &e = a.e;
  const int lane = threadIdx.x & 31;
  if constexpr (EPI == GB_EPI_PLAIN) {
    int r = rbk * 32 + lane;
    if (r < a.rows) e.y[r] = y0;
  } else if constexpr (EPI == GB_EPI_RESID) {
    // cpu.Add, backend/cpu/cpu.go:60; the sums of squares feed the next RMSNorm
    int r = rbk * 32 + lane;
    float xn = e.x[r] + y0;
    e.x[r] = xn;
    float ss = gb_warp_sum(xn * xn);
    if (lane == 0) e.ssq[rbk] = ss;
  } else if constexpr (EPI == GB_EPI_SWIGLU) {  // cpu.SiluMul, backend/cpu/cpu.go:53
    float g = y0, u = y1;
    float ex = (float)exp(-(double)g);
    e.y[rbk * 32 + lane] = g / (1.f + ex) * u;
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
      const double *cs = rope_row + (size_t)j * 2;  // row `pos` of the table, staged at kernel start
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
  } else if constexpr (EPI == GB_EPI_PARTIAL) {
    // this rank's partial of rows r into its own slot as tagged words
    // ((step + 1) << 32 | float bits): the other ranks read them over NVLink
    // and know each word is this step's by its tag, so no fence, counter or
    // flag is needed here
    const GbPeer &P = e.peer;
    const unsigned long long tag = (unsigned long long)(__ldcg(P.epoch) + 1u) << 32;
    gb_st_relaxed_sys_u64(P.my_tbuf + (size_t)e.peer_slot * P.dim + rbk * 32 + lane,
                          tag | (unsigned long long)__float_as_uint(y0));
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
        if (e.peer_slot >= 0) {
          // tensor parallel: this rank's key into its own slot, then the flag
          const GbPeer &P = e.peer;
          *(unsigned long long *)(P.my_buf + (size_t)e.peer_slot * P.dim) = k;
          gb_st_release_sys(P.my_flag + e.peer_slot, *P.epoch + 1u);
        }
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

template <int TA, int TB>
GB_DEV float decode(int ty, const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xsum, const uint2 *sl, float xs) {
  if (TA == TB || ty == TA) return sb_dot<TA>(st, lane, xa, xb, xc, xsum, sl, xs);
  return sb_dot<TB>(st, lane, xa, xb, xc, xsum, sl, xs);
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
// against the staged activation and release each unit's slot through the
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
  const int nsb = a.nsb, LK = p.lk, K = 1 << LK, NS = p.nstage;
  const unsigned U = p.units, G = gridDim.x, b = blockIdx.x;
  const unsigned cu0 = ubeg(U, G, b), cu1 = ubeg(U, G, b + 1);
  const unsigned nst = (cu1 - cu0 + (unsigned)K - 1) >> LK;  // stages of this CTA

  // shared memory: [NS] stages | staged activation [XS] | 2 x [W][64] segment partials
  uint8_t *ring = smem;
  const int XS = p.xs_max;
  uint8_t *xbase = smem + (size_t)NS * p.stage_bytes;
  uint32_t *xa_s = (uint32_t *)xbase;
  uint32_t *xb_s = xa_s + XS * 64;
  uint32_t *xc_s = xb_s + XS * 64;
  float *xsum_s = (float *)(xc_s + XS * 64);
  uint2 *sl_s = (uint2 *)(xsum_s + XS * 16);
  float *xs_s = (float *)(sl_s + XS * 16);
  float *psum = xs_s + ((XS + 3) & ~3);  // [2][kPend][W][64]
  float *wn_s = psum + 2 * kPend * W * 64;                    // [XS][256] norm weights (aux_w)
  double *rope_s = (double *)(wn_s + (p.aux_w ? XS * 256 : 0));  // RoPE row (aux_rope doubles)
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ __align__(8) uint64_t aux;  // norm weights and RoPE row landed
  __shared__ double red[W];
  __shared__ float inv_s;

  // 0. let the next kernel's CTAs start (they stream their weights meanwhile)
  gb_grid_dep_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      gb_mbar_init(&full[s], 1);
      gb_mbar_init(&empty[s], (uint32_t)K);
    }
    gb_mbar_init(&aux, 1);
    gb_mbar_fence_init();
  }
  __syncthreads();
  // super-blocks of activation this CTA touches: [sbf, sbf + nsbs) mod nsb
  const int half = p.half;
  const unsigned upr = (unsigned)p.upr;
  const unsigned su0 = half ? cu0 >> 1 : cu0, su1 = half ? ((cu1 - 1) >> 1) + 1 : cu1;  // super-block units
  const int nsbs = (su1 - su0) >= (unsigned)nsb ? nsb : (int)(su1 - su0);
  const int sbf = (int)(su0 % (unsigned)nsb);
  const bool use_aux = p.aux_w || p.aux_rope;

  if (warp == W) {
    // 1. producer: weights do not depend on the previous kernel. First the
    // norm weights of the staged super-blocks and the RoPE row of `pos`
    // (constant tables that the weight stream evicts from L2 every token, so
    // reading them in the prologue would be a DRAM round trip ahead of the
    // activation's L2 loads); `pos` is set before the step starts.
    if (lane == 0) {
      if (use_aux) {
        const int n1 = min(nsbs, nsb - sbf);
        int pos = 0;
        if (p.aux_rope) pos = min(max(*a.e.pos, 0), a.e.max_len - 1);
        gb_mbar_expect_tx(&aux, (uint32_t)((p.aux_w ? nsbs * 1024 : 0) + p.aux_rope * 8));
        if (p.aux_w) {
          gb_bulk_g2s(wn_s, a.in_w + (size_t)sbf * 256, (uint32_t)n1 * 1024u, &aux);
          if (nsbs > n1) gb_bulk_g2s(wn_s + (size_t)n1 * 256, a.in_w, (uint32_t)(nsbs - n1) * 1024u, &aux);
        }
        if (p.aux_rope)
          gb_bulk_g2s(rope_s, a.e.rope_cs + (size_t)pos * p.aux_rope, (uint32_t)p.aux_rope * 8u, &aux);
      }
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
        const unsigned j0 = cu0 + (k << LK), j1 = min(cu1, j0 + (unsigned)K);
        const size_t o0 = unit_off<TA, TB>(p, j0), o1 = unit_off<TA, TB>(p, j1);
        gb_mbar_expect_tx(&full[s], (uint32_t)(o1 - o0));
        gb_bulk_g2s(ring + (size_t)s * p.stage_bytes, a.w + o0, (uint32_t)(o1 - o0), &full[s]);
      }
      // the copies still in flight land (bounded) before the CTA exits
      for (unsigned j = k > (unsigned)NS ? k - NS : 0; j < k; j++)
        (void)gb_mbar_wait(&full[j % NS], (j / NS) & 1);
      if (use_aux) (void)gb_mbar_wait(&aux, 0);
    }
    return;
  }

  // 2. stage the activation of the super-blocks this CTA touches. The input
  // is a float vector from the preceding kernel; an RMS-normalised input is
  // z = (x * inv) * w with inv = 1/sqrt(sum x^2 / n + eps) from per-32 sums of
  // squares (cpu.RMSNorm, backend/cpu/cpu.go:17: float64 sum, float32 products).
  // Per super-block: s = max|z| / 127 and three int8 limbs per element,
  // z ~ s*(a + b/254 + c/254^2) (error below 2^-21 of the block maximum).
  constexpr int CT = W * 32;
  const int tid = threadIdx.x;
  gb_grid_dep_wait();
  // this warp's first super-block of x is loaded with the sums of squares
  // (it does not depend on them): one L2 round trip instead of two
  float4 x0p = make_float4(0.f, 0.f, 0.f, 0.f), x1p = x0p;
  if (warp < nsbs) {
    int sb = sbf + warp;
    if (sb >= nsb) sb -= nsb;
    x0p = __ldcg((const float4 *)(a.in_x + sb * 256 + lane * 8));
    x1p = __ldcg((const float4 *)(a.in_x + sb * 256 + lane * 8 + 4));
  }
  float inv = 1.f;
  if (a.in_ssq) {
    double ss = 0;
    for (int g = tid; g < nsb * 8; g += CT) ss += (double)__ldcg(a.in_ssq + g);
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
    inv = inv_s;
  }
  bool timeout = use_aux && !gb_mbar_wait(&aux, 0);
  for (int ls = warp; ls < nsbs; ls += W) {
    int sb = sbf + ls;
    if (sb >= nsb) sb -= nsb;
    const int e0 = sb * 256 + lane * 8;
    float z[8];
    {
      const bool first = ls == warp;
      const float4 x0 = first ? x0p : __ldcg((const float4 *)(a.in_x + e0));
      const float4 x1 = first ? x1p : __ldcg((const float4 *)(a.in_x + e0 + 4));
      z[0] = x0.x; z[1] = x0.y; z[2] = x0.z; z[3] = x0.w;
      z[4] = x1.x; z[5] = x1.y; z[6] = x1.z; z[7] = x1.w;
      if (a.in_w) {
        const float4 *wq = (const float4 *)(wn_s + (size_t)ls * 256 + lane * 8);
        const float4 w0 = wq[0], w1 = wq[1];
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) z[i] = __fmul_rn(__fmul_rn(z[i], inv), wv[i]);
      }
    }
    float m = 0.f, zs = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      m = fmaxf(m, fabsf(z[i]));
      zs += z[i];
    }
    m = gb_warp_max(m);
    const float r = m > 0.f ? 127.f / m : 0.f;
    uint32_t wa[2] = {0u, 0u}, wb[2] = {0u, 0u}, wc[2] = {0u, 0u};
    int sa = 0, sbs = 0, sc = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float t = z[i] * r;
      const float fa = rintf(t), r1 = (t - fa) * 254.f, fb = rintf(r1), fc = rintf((r1 - fb) * 254.f);
      const int ia = (int)fa, ib = (int)fb, ic = (int)fc;
      sa += ia;
      sbs += ib;
      sc += ic;
      wa[i >> 2] |= (uint32_t)(ia & 0xFF) << (8 * (i & 3));
      wb[i >> 2] |= (uint32_t)(ib & 0xFF) << (8 * (i & 3));
      wc[i >> 2] |= (uint32_t)(ic & 0xFF) << (8 * (i & 3));
    }
    ((uint2 *)(xa_s + ls * 64))[lane] = make_uint2(wa[0], wa[1]);
    ((uint2 *)(xb_s + ls * 64))[lane] = make_uint2(wb[0], wb[1]);
    ((uint2 *)(xc_s + ls * 64))[lane] = make_uint2(wc[0], wc[1]);
    // lanes 2i and 2i+1 hold 16-group i
    zs += __shfl_xor_sync(0xffffffffu, zs, 1);
    sa += __shfl_xor_sync(0xffffffffu, sa, 1);
    sbs += __shfl_xor_sync(0xffffffffu, sbs, 1);
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    if ((lane & 1) == 0) {
      xsum_s[ls * 16 + (lane >> 1)] = zs;
      sl_s[ls * 16 + (lane >> 1)] =
          make_uint2(((uint32_t)sa & 0xFFFFu) | ((uint32_t)sbs << 16), (uint32_t)sc & 0xFFFFu);
    }
    if (lane == 0) xs_s[ls] = m / 127.f;
  }
  consumers_sync<W>();

  // 3. units round-robin over the warps, segment by segment. Cursors advance
  // by W units per step: stage k = j >> LK (K is a power of two), ring slot
  // s = k mod NS with the phase parity ph, super-block usb = u mod nsb.
  const size_t sbb_a = (size_t)gb_tiled_sb_bytes(TA);
  const unsigned dk = (unsigned)W >> LK;  // stages per step (K <= W)
  // A warp takes every dk-th stage. When dk does not divide NS, the stage
  // that last used slot s (k - NS) was other warps', and may still be in
  // flight when this warp gets to stage k: a parity wait on full[s] for k
  // alone would then see the completed phase before k - NS (same parity)
  // and read early. So such a warp first waits until slot s was released
  // after stage k - NS: phase (k - NS) of empty[s], parity ph ^ 1. Its
  // consumers arrive there only after full[s] completed k - NS, and the
  // next phase of empty[s] cannot complete before this warp arrives, so the
  // parity is unambiguous. That needs stage k - NS to have been issued: the
  // launcher keeps dk <= NS, so this warp's own stage k - dk >= k - NS has
  // landed, and stages are issued in order.
  const bool prewait = (unsigned)NS % dk != 0u;
  unsigned j = (unsigned)warp;  // this warp's next unit (CTA-relative)
  unsigned k = j >> LK;
  int s = (int)(k % (unsigned)NS);
  uint32_t ph = (k / (unsigned)NS) & 1u;
  unsigned usb = ((cu0 + j) >> half) % (unsigned)nsb;
  const unsigned dsb = (unsigned)W >> half;              // super-blocks per step
  const int hw = half ? (int)((cu0 + j) & 1u) : 0;        // gate (0) or up (1) rows of this warp (W even)
  int nseg = 0;
  unsigned batch_s0 = cu0;  // first unit of the current batch of segments
  for (unsigned s0 = cu0; s0 < cu1; nseg++) {
    const int rbk = (int)(s0 / upr);
    const unsigned s1 = min(cu1, (unsigned)(rbk + 1) * upr);
    const int ty = rbk < a.split_tile ? TA : TB;
    float acc0 = 0.f;
    for (; cu0 + j < s1;) {
      const unsigned u = cu0 + j;
      if (prewait && k >= (unsigned)NS && !timeout && !gb_mbar_wait(&empty[s], ph ^ 1u)) timeout = true;
      if (!timeout && !gb_mbar_wait(&full[s], ph)) timeout = true;
      if (!timeout) {
        int ls = (int)usb - sbf;
        if (ls < 0) ls += nsb;
        const uint32_t *xa = xa_s + ls * 64, *xb = xb_s + ls * 64, *xc = xc_s + ls * 64;
        const float *xsum = xsum_s + ls * 16;
        const uint2 *sl = sl_s + ls * 16;
        const float xs = xs_s[ls];
        const size_t off = TA == TB ? (size_t)(j & (unsigned)(K - 1)) * (size_t)p.rb * sbb_a
                                    : unit_off<TA, TB>(p, u) - unit_off<TA, TB>(p, cu0 + (k << LK));
        const uint8_t *st = ring + (size_t)s * p.stage_bytes + off;
        acc0 += decode<TA, TB>(ty, st, lane, xa, xb, xc, xsum, sl, xs);
      }
      __syncwarp();
      if (lane == 0) gb_mbar_arrive(&empty[s]);
      j += W;
      k += dk;
      s += (int)dk;
      while (s >= NS) {
        s -= NS;
        ph ^= 1u;
      }
      usb += dsb;
      while (usb >= (unsigned)nsb) usb -= nsb;
    }
    // this warp's partials of segment nseg go to slot nseg % kPend of the
    // batch's half of psum; a batch (kPend segments, or the end of the range)
    // ends with one barrier, after which each pending segment is reduced by
    // its own warp. A half is written again only after the next batch's
    // barrier, which the reducers of this batch pass first.
    const int slot = nseg % kPend, half = (nseg / kPend) & 1;
    if (slot == 0) batch_s0 = s0;
    float *ps = psum + (size_t)(half * kPend + slot) * W * 64;
    ps[warp * 64 + hw * 32 + lane] = acc0;  // the other family's half stays zero
    ps[warp * 64 + (1 - hw) * 32 + lane] = 0.f;
    s0 = s1;
    if (slot == kPend - 1 || s0 >= cu1) {
      consumers_sync<W>();
      for (int q = 0; q <= slot; q++) {
        const int seg = nseg - slot + q;
        if (warp != seg % W) continue;  // reducer of segment seg (sum in warp order)
        // segments after the batch's first start on row-block boundaries
        const unsigned t0 = q == 0 ? batch_s0 : (batch_s0 / upr + (unsigned)q) * upr;
        const int rbq = (int)(t0 / upr);
        const unsigned t1 = min(cu1, (unsigned)(rbq + 1) * upr);
        const float *pq = psum + (size_t)(half * kPend + q) * W * 64;
        float y0 = 0.f, y1 = 0.f;
        for (int w2 = 0; w2 < W; w2++) {
          y0 += pq[w2 * 64 + lane];
          y1 += pq[w2 * 64 + 32 + lane];
        }
        const unsigned R0 = (unsigned)rbq * upr, R1 = R0 + upr;
        if (t0 == R0 && t1 == R1) {
          epilogue<EPI>(p, rbq, y0, y1, rope_s);
        } else {
          // the row-block continues in another CTA: global partial per CTA
          const int which = cu0 >= R0 ? 0 : 1;
          float *gslot = a.e.part + ((size_t)b * 2 + which) * 64;
          gslot[lane] = y0;
          gslot[32 + lane] = y1;
          __threadfence();
          __syncwarp();
          unsigned done = 0;
          if (lane == 0) done = atomicAdd(a.e.tile_counter + rbq, t1 - t0) + (t1 - t0);
          done = __shfl_sync(0xffffffffu, done, 0);
          if (done == upr) {
            __threadfence();
            const unsigned bf = cta_of_unit(U, G, R0), bl = cta_of_unit(U, G, R1 - 1);
            float z0 = 0.f, z1 = 0.f;
            for (unsigned b2 = bf; b2 <= bl; b2++) {
              const unsigned c0 = ubeg(U, G, b2), c1 = ubeg(U, G, b2 + 1);
              if (c0 == c1) continue;
              const float *sl2 = a.e.part + ((size_t)b2 * 2 + (c0 >= R0 ? 0 : 1)) * 64;
              z0 += __ldcg(sl2 + lane);
              z1 += __ldcg(sl2 + 32 + lane);
            }
            if (lane == 0) a.e.tile_counter[rbq] = 0u;
            epilogue<EPI>(p, rbq, z0, z1, rope_s);
          }
        }
      }
    }
  }
  if (timeout && lane == 0 && a.e.err) atomicOr(a.e.err, GB_DEVERR_TIMEOUT);
}

// ---- unquantized weights (F16 / F32 matrices) ------------------------------
// model.Linear's MatVecF16 / MatVecF32 (model/model.go:108-117). One CTA of
// 8 warps per row-block (or gate/up pair), so no row-block is split: the
// input is staged in shared memory as floats (RMSNorm applied as in the
// quantized path), warp w takes super-blocks w, w + 8, ... with lane = row
// and several 16-byte streaming loads in flight, and the warps' sums are
// added in warp order before the same fused epilogue.
// Element tag for bfloat16 weights (16 bits, decoded by widening).
struct Bf16 {
  uint16_t bits;
};
template <typename T>
struct TW_BF16 {
  static constexpr bool value = false;
};
template <>
struct TW_BF16<Bf16> {
  static constexpr bool value = true;
};

template <typename TW, int EPI>
__global__ void __launch_bounds__(256) gemv_float_kernel(const Kp p) {
  extern __shared__ __align__(16) float fz[];  // [nsb*256] input, then [8][64] partials
  __shared__ double red[8];
  __shared__ float inv_s;
  const GbGemvArgs &a = p.a;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
  const int nsb = a.nsb, n = nsb * 256, rbk = blockIdx.x, G = p.half ? 2 : 1;
  gb_grid_dep_launch();
  gb_grid_dep_wait();
  float inv = 1.f;
  if (a.in_ssq) {
    double ss = 0;
    for (int g = tid; g < nsb * 8; g += 256) ss += (double)__ldcg(a.in_ssq + g);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      double t = 0;
      for (int w2 = 0; w2 < 8; w2++) t += red[w2];
      inv_s = (float)(1.0 / sqrt(t / (double)n + (double)a.eps));
    }
    __syncthreads();
    inv = inv_s;
  }
  for (int i = tid * 4; i < n; i += 256 * 4) {
    float4 x = __ldcg((const float4 *)(a.in_x + i));
    if (a.in_w) {
      const float4 w = __ldg((const float4 *)(a.in_w + i));
      x = make_float4(__fmul_rn(__fmul_rn(x.x, inv), w.x), __fmul_rn(__fmul_rn(x.y, inv), w.y),
                      __fmul_rn(__fmul_rn(x.z, inv), w.z), __fmul_rn(__fmul_rn(x.w, inv), w.w));
    }
    *(float4 *)(fz + i) = x;
  }
  __syncthreads();
  constexpr int EPU = 16 / (int)sizeof(TW);  // elements per 16-byte unit
  constexpr int UPB = 256 / EPU;              // units per row and super-block
  const size_t sbb = (size_t)32 * UPB * 16;
  float acc[2] = {0.f, 0.f};
  for (int sb = warp; sb < nsb; sb += 8) {
    for (int g = 0; g < G; g++) {
      const uint8_t *blk = a.w + (((size_t)rbk * nsb + sb) * G + g) * sbb + lane * 16;
      const float *zs = fz + sb * 256;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
      for (int u = 0; u < UPB; u++) {
        const uint4 v = gb_ld_stream16(blk + (size_t)u * 512);
        const float4 z0 = *(const float4 *)(zs + u * EPU);
        if constexpr (EPU == 8) {
          const float4 z1 = *(const float4 *)(zs + u * EPU + 4);
          float2 f0, f1, f2, f3;
          if constexpr (sizeof(TW) == 2 && TW_BF16<TW>::value) {  // bf16: the high half of a float
            f0 = make_float2(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u));
            f1 = make_float2(__uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
            f2 = make_float2(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u));
            f3 = make_float2(__uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
          } else {
            f0 = __half22float2(*(const __half2 *)&v.x);
            f1 = __half22float2(*(const __half2 *)&v.y);
            f2 = __half22float2(*(const __half2 *)&v.z);
            f3 = __half22float2(*(const __half2 *)&v.w);
          }
          s0 = fmaf(f0.x, z0.x, fmaf(f0.y, z0.y, fmaf(f1.x, z0.z, fmaf(f1.y, z0.w, s0))));
          s1 = fmaf(f2.x, z1.x, fmaf(f2.y, z1.y, fmaf(f3.x, z1.z, fmaf(f3.y, z1.w, s1))));
        } else {
          s0 = fmaf(__uint_as_float(v.x), z0.x, fmaf(__uint_as_float(v.y), z0.y, s0));
          s1 = fmaf(__uint_as_float(v.z), z0.z, fmaf(__uint_as_float(v.w), z0.w, s1));
        }
      }
      acc[g] += s0 + s1;
    }
  }
  float *ps = fz + n;
  ps[warp * 64 + lane] = acc[0];
  ps[warp * 64 + 32 + lane] = acc[1];
  __syncthreads();
  if (warp == 0) {
    float y0 = 0.f, y1 = 0.f;
    for (int w2 = 0; w2 < 8; w2++) {
      y0 += ps[w2 * 64 + lane];
      y1 += ps[w2 * 64 + 32 + lane];
    }
    const double *rope_row = nullptr;
    if constexpr (EPI == GB_EPI_QKV) {
      const int pos = min(max(*a.e.pos, 0), a.e.max_len - 1);
      rope_row = a.e.rope_cs + (size_t)pos * a.e.head_dim;
    }
    epilogue<EPI>(p, rbk, y0, y1, rope_row);
  }
}

template <typename TW>
KernelFnF pick_float(int epi) {
  switch (epi) {
    case GB_EPI_PLAIN: return gemv_float_kernel<TW, GB_EPI_PLAIN>;
    case GB_EPI_QKV: return gemv_float_kernel<TW, GB_EPI_QKV>;
    case GB_EPI_RESID: return gemv_float_kernel<TW, GB_EPI_RESID>;
    case GB_EPI_SWIGLU: return gemv_float_kernel<TW, GB_EPI_SWIGLU>;
    case GB_EPI_LOGITS: return gemv_float_kernel<TW, GB_EPI_LOGITS>;
    case GB_EPI_PARTIAL: return gemv_float_kernel<TW, GB_EPI_PARTIAL>;
  }
  return nullptr;
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

// Dynamic shared memory: ring stages, then per staged super-block the limb
// planes (3 x 256 B), 16 sums (64 B) and 16 packed limb sums (128 B), the
// scales (padded to 4 floats), then 2 x kPend x [warps][64] segment partials.
size_t gemv_smem(int warps, int nstage, int stage_bytes, int xs_max, int aux_w, int aux_rope) {
  return (size_t)nstage * stage_bytes + (size_t)xs_max * (3 * 256 + 64 + 128) +
         (size_t)((xs_max + 3) & ~3) * 4 + (size_t)2 * kPend * warps * 64 * 4 + (aux_w ? (size_t)xs_max * 1024 : 0) +
         (size_t)aux_rope * 8;
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
    case GB_EPI_PARTIAL: return gemv_kernel<TA, TB, GB_EPI_PARTIAL, W>;
  }
  return nullptr;
}

template <int W>
KernelFn pick_w(int ta, int tb, int epi) {
  if (ta == tb) {
    if (ta == GB_T_Q4_K) return pick_epi<GB_T_Q4_K, GB_T_Q4_K, W>(epi);
    if (ta == GB_T_Q6_K) return pick_epi<GB_T_Q6_K, GB_T_Q6_K, W>(epi);
    if (ta == GB_T_Q5_K) return pick_epi<GB_T_Q5_K, GB_T_Q5_K, W>(epi);
    if (ta == GB_T_Q4_0) return pick_epi<GB_T_Q4_0, GB_T_Q4_0, W>(epi);
    if (ta == GB_T_Q8_0) return pick_epi<GB_T_Q8_0, GB_T_Q8_0, W>(epi);
  } else if (ta == GB_T_Q4_K && tb == GB_T_Q6_K && epi == GB_EPI_QKV) {
    return gemv_kernel<GB_T_Q4_K, GB_T_Q6_K, GB_EPI_QKV, W>;
  } else if (ta == GB_T_Q6_K && tb == GB_T_Q4_K && epi == GB_EPI_QKV) {
    return gemv_kernel<GB_T_Q6_K, GB_T_Q4_K, GB_EPI_QKV, W>;
  } else if (ta == GB_T_Q5_K && tb == GB_T_Q6_K && epi == GB_EPI_QKV) {  // Q5_K_M: q, k Q5_K, v Q6_K
    return gemv_kernel<GB_T_Q5_K, GB_T_Q6_K, GB_EPI_QKV, W>;
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

GbGemvPlan gb_gemv_plan(int ntiles, int nsb, int epi, int nsm) {
  GbGemvPlan p;
  p.rb = 1;
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

namespace {
int gemv_float_launch(const GbGemvArgs &a, cudaStream_t st, bool pdl) {
  Kp p;
  p.a = a;
  p.half = a.epi == GB_EPI_SWIGLU ? 1 : 0;
  if (p.half && a.ntiles % 2) return gb_fail(GB_ERR_INVALID, "gpu: gemv: tiles not paired");
  if (a.split_tile < a.ntiles && a.type_b != a.type_a)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: unquantized and quantized rows in one matrix");
  p.nrb = p.half ? a.ntiles / 2 : a.ntiles;
  KernelFnF fn = a.type_a == GB_T_F16    ? pick_float<__half>(a.epi)
                 : a.type_a == GB_T_BF16 ? pick_float<Bf16>(a.epi)
                                         : pick_float<float>(a.epi);
  if (!fn) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: epilogue %d", a.epi);
  const size_t smem = sizeof(float) * ((size_t)a.nsb * 256 + 8 * 64);
  static KernelFnF opted[18];
  static int nopted = 0;
  bool seen = false;
  for (int i = 0; i < nopted; i++) seen = seen || opted[i] == fn;
  if (!seen) {
    GB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin() - 4096),
            "gpu: gemv: shared memory attribute");
    if (nopted < 18) opted[nopted++] = fn;
  }
  if ((long long)smem > smem_optin() - 4096)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: %d input columns exceed shared memory", a.nsb * 256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.nrb);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GB_CUDA(cudaLaunchKernelEx(&cfg, fn, p), "gpu: gemv launch (unquantized weights)");
  return GB_OK;
}
}  // namespace

int gb_gemv_launch(const GbGemvArgs &a, const GbGemvPlan &plan, cudaStream_t st, bool pdl) {
  if (a.nsb <= 0 || a.ntiles <= 0) return gb_fail(GB_ERR_INVALID, "gpu: gemv: empty matrix");
  if (gb_float_type(a.type_a)) return gemv_float_launch(a, st, pdl);
  Kp p;
  p.a = a;
  p.rb = 1;
  p.half = a.epi == GB_EPI_SWIGLU ? 1 : 0;
  p.aux_w = a.in_w != nullptr ? 1 : 0;
  p.aux_rope = a.epi == GB_EPI_QKV ? a.e.head_dim : 0;
  if (p.half && a.ntiles % 2) return gb_fail(GB_ERR_INVALID, "gpu: gemv: tiles not paired");
  const int ta = a.type_a, tb = a.split_tile < a.ntiles ? a.type_b : a.type_a;
  p.a.type_b = tb;
  if (p.half && ta != tb) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: gate/up types differ");
  p.nrb = p.half ? a.ntiles / 2 : a.ntiles;
  p.upr = p.half ? 2 * a.nsb : a.nsb;
  p.units = (unsigned)p.nrb * (unsigned)p.upr;
  const int ub = p.rb * std::max(gb_tiled_sb_bytes(ta), gb_tiled_sb_bytes(tb));  // largest unit
  // SMs a launch spreads over (GB_GEMV_SMS overrides, for sweeps)
  int nsm = sms();
  if (const char *e = getenv("GB_GEMV_SMS")) nsm = std::max(1, std::min(nsm, atoi(e)));
  const long long cap = smem_optin();
  static const char *epi_names[] = {"PLAIN", "QKV", "RESID", "SWIGLU", "LOGITS", "PARTIAL"};
  // Paired launch: two 8-warp CTAs per SM, so that a matrix of up to twice as
  // many row-blocks as SMs runs one row-block per CTA with no split (and no
  // cross-CTA combine at its end). Used for short row-blocks (at most 16
  // units, e.g. the 8B's q|k|v: 192 row-blocks of 16 units, measured 2 %
  // faster per token); GB_GEMV_PAIR_<KIND> / GB_GEMV_PAIR = 0 or 1 override.
  bool pair = p.nrb > nsm && p.nrb <= 2 * nsm && p.upr <= 16;
  {
    char key[64];
    snprintf(key, sizeof key, "GB_GEMV_PAIR_%s", epi_names[a.epi]);
    const char *e = getenv(key);
    if (!e) e = getenv("GB_GEMV_PAIR");
    if (e) pair = atoi(e) == 1;
  }
  const long long slots = pair ? 2LL * nsm : nsm;
  long long grid = p.nrb <= slots ? p.nrb : std::min<long long>(slots, p.units);
  if (grid * 128 > (long long)gb_gemv_scratch_floats(a.ntiles, plan)) grid = gb_gemv_scratch_floats(a.ntiles, plan) / 128;
  const int upc = (int)((p.units + grid - 1) / grid);  // units per CTA (at most)
  const int xs = std::min(a.nsb, (p.half ? upc / 2 + 1 : upc) + 1);  // super-blocks a CTA touches
  // consumer warps per CTA: 16 (a whole SM) or 8 (half an SM); GB_GEMV_WARPS
  // overrides. The ring holds at least one unit per consumer warp; when that
  // minimum and the staged activation of a very wide input (e.g. the 70B's
  // 28,672-column down projection with 6.7 KB Q6_K units) exceed shared
  // memory with 16 warps, the launch uses 8 and all of shared memory.
  int warps = pair ? 8 : 16;
  if (const char *e = getenv("GB_GEMV_WARPS")) warps = atoi(e) == 8 ? 8 : 16;
  bool wide = false;
  if (warps == 16 && (long long)gemv_smem(16, 0, 0, xs, p.aux_w, p.aux_rope) + 16LL * ub > cap - 1024) {
    warps = 8;
    wide = true;
  }
  KernelFn fn = pick(ta, tb, a.epi, warps);
  if (!fn) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: types %d/%d with epilogue %d", ta, tb, a.epi);
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
  int fk = 0, fs = 0;
  {
    char key[64];
    snprintf(key, sizeof key, "GB_GEMV_RING_%s", epi_names[a.epi]);
    const char *e = getenv(key);
    if (!e) e = getenv("GB_GEMV_RING");
    if (e && sscanf(e, "%d,%d", &fk, &fs) != 2) fk = fs = 0;
  }
  long long budget = wide ? cap - 2048 : warps == 8 ? 113 * 1024 : 220 * 1024;
  if (const char *e = getenv("GB_SMEM_BUDGET")) budget = atoll(e);
  const long long room = cap - static_smem;
  const long long fixed = (long long)gemv_smem(warps, 0, 0, xs, p.aux_w, p.aux_rope);
  // K: a power of two, at most the consumer warps (each warp then takes one
  // unit every warps/K stages), about 36 KB per stage, at most the units a
  // CTA owns
  auto pow2_floor = [](int v) {
    int r = 1;
    while (r * 2 <= v) r *= 2;
    return r;
  };
  int K = pow2_floor(std::max(1, std::min(warps, (36 * 1024 + ub / 2) / ub)));
  K = std::min(K, pow2_floor(std::max(1, upc)));
  int ns = 0;
  // A consumer warp takes every (warps/K)-th stage, so the ring must hold at
  // least warps/K stages: then a warp's own previous stage bounds the phase
  // of the slot it waits on next (gemv_kernel, step 3).
  if (fk > 0 && fk <= warps && (fk & (fk - 1)) == 0 && fs >= 2 && fs <= kMaxStages && warps / fk <= fs &&
      fixed + (long long)fs * fk * ub <= room) {
    K = fk;
    ns = fs;
  } else {
    for (;; K /= 2) {
      ns = (int)std::min<long long>(kMaxStages, (budget - fixed) / ((long long)K * ub));
      if (ns >= 2 || K == 1) break;
    }
    if (ns < 2) ns = 2;
    while (warps / K > ns && (upc + K - 1) / K > ns && K < warps) {
      K *= 2;
      ns = (int)std::max<long long>(2, std::min<long long>(kMaxStages, (budget - fixed) / ((long long)K * ub)));
    }
  }
  int lk = 0;
  while ((1 << lk) < K) lk++;
  p.lk = lk;
  p.nstage = ns;
  p.stage_bytes = (K * ub + 127) / 128 * 128;
  p.xs_max = xs;
  const size_t smem = gemv_smem(warps, ns, p.stage_bytes, xs, p.aux_w, p.aux_rope);
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
