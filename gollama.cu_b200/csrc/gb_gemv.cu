// gb_gemv.cu -- batch-1 quantized matrix-vector products on the tiled layout
// (gb_formats.h), with fused epilogues for the decode step.
//
// Replaces kernels.MatVecQ4_0 / MatVecQ4K / MatVecQ6K (kernels/quantmv.go:18-136)
// on the model path. Design:
//  * Work is the list of units (row-block, super-block); a row-block is one
//    32-row tile, or a gate/up tile pair for the SwiGLU epilogue. Every warp
//    of the persistent grid takes one contiguous range of units (stream-K),
//    so all SMs stay busy whatever the matrix shape and no wave is partial.
//  * Each unit's sb-block (4608 or 6720 contiguous bytes) is brought into a
//    per-warp shared-memory ring by one 1-D TMA bulk copy completing on an
//    mbarrier; the copies of the next units are in flight while the warp
//    decodes the current one. Lane l of the warp owns row l of the tile.
//  * The activation arrives as a limb pack (gb_device.cuh): three int8
//    limbs per element, so the 4-bit / 6-bit quants meet the activation in
//    dp4a (4 products per instruction, exact int32 sums), and float math is
//    only needed once per 16- or 32-element sub-block for the ggml scales.
//  * A row-block split between warps is finished by the warp whose atomic
//    count completes it; it sums the partials in warp order (deterministic)
//    and runs the epilogue. Counters are reset by that warp, so the kernel
//    can be replayed from a CUDA graph.
#include <math.h>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr float kL1 = 1.f / 254.f;
constexpr float kL2 = 1.f / 64516.f;

GB_DEV float byte_f(uint32_t w, int i) { return (float)((w >> (8 * i)) & 0xFFu); }

// ---- per-super-block decode + dot products. `st` is the sb-block in shared
// memory; xa/xb/xc are the limb planes (as 32-bit words) of the block's 256
// activation elements, xs the 8 group scales and xsum the 16 half-group sums.

// Q4_K: quant/quant.go:97 layout; kernels/quantmv.go:66 factorisation
// sum = d*sum_j sc_j*(q.x)_j - dmin*sum_j m_j*(sum x)_j.
GB_DEV float sb_q4k(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  uint4 h = u[lane];
  float d = gb_half_to_float((uint16_t)(h.x & 0xFFFFu));
  float dmin = gb_half_to_float((uint16_t)(h.x >> 16));
  uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
  uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  float tq = 0.f, tm = 0.f;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint4 q0 = u[(1 + 2 * c) * 32 + lane], q1 = u[(2 + 2 * c) * 32 + lane];
    uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint4 *pa = (const uint4 *)(xa + 16 * c), *pb = (const uint4 *)(xb + 16 * c),
                *pc = (const uint4 *)(xc + 16 * c);
    int A0 = 0, B0 = 0, C0 = 0, A1 = 0, B1 = 0, C1 = 0;
#pragma unroll
    for (int v = 0; v < 2; v++) {
      uint4 la = pa[v], lb = pb[v], lc = pc[v], ha = pa[2 + v], hb = pb[2 + v], hc = pc[2 + v];
      uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
               c4[4] = {lc.x, lc.y, lc.z, lc.w};
      uint32_t A4[4] = {ha.x, ha.y, ha.z, ha.w}, B4[4] = {hb.x, hb.y, hb.z, hb.w},
               C4[4] = {hc.x, hc.y, hc.z, hc.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        uint32_t w = qw[4 * v + k];
        uint32_t lo = w & 0x0F0F0F0Fu, hi = w & 0xF0F0F0F0u;
        A0 = gb_dp4a_us(lo, a4[k], A0);
        B0 = gb_dp4a_us(lo, b4[k], B0);
        C0 = gb_dp4a_us(lo, c4[k], C0);
        A1 = gb_dp4a_us(hi, A4[k], A1);
        B1 = gb_dp4a_us(hi, B4[k], B1);
        C1 = gb_dp4a_us(hi, C4[k], C1);
      }
    }
    float S0 = (float)A0 + (float)B0 * kL1 + (float)C0 * kL2;
    float S1 = ((float)A1 + (float)B1 * kL1 + (float)C1 * kL2) * 0.0625f;
    const int j0 = 2 * c, j1 = 2 * c + 1;
    float sc0 = byte_f(j0 < 4 ? sc03 : sc47, j0 & 3), sc1 = byte_f(j1 < 4 ? sc03 : sc47, j1 & 3);
    float m0 = byte_f(j0 < 4 ? m03 : m47, j0 & 3), m1 = byte_f(j1 < 4 ? m03 : m47, j1 & 3);
    tq += sc0 * (xs[j0] * S0) + sc1 * (xs[j1] * S1);
    tm += m0 * (xsum[2 * j0] + xsum[2 * j0 + 1]) + m1 * (xsum[2 * j1] + xsum[2 * j1 + 1]);
  }
  return d * tq - dmin * tm;
}

// Q6_K: quant/quant.go:114 layout; y = d*sc*(q-32) over 16-element sub-blocks.
GB_DEV float sb_q6k(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  uint4 scv = u[12 * 32 + lane];
  const int8_t *sc8 = (const int8_t *)&scv;
  float d = gb_half_to_float(((const uint16_t *)(st + 13 * 512))[lane]);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 2; c++) {
    uint4 l0 = u[(4 * c + 0) * 32 + lane], l1 = u[(4 * c + 1) * 32 + lane];
    uint4 l2 = u[(4 * c + 2) * 32 + lane], l3 = u[(4 * c + 3) * 32 + lane];
    uint4 h0 = u[(8 + 2 * c) * 32 + lane], h1 = u[(9 + 2 * c) * 32 + lane];
    uint32_t ql[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                       l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
    uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int is = 0; is < 2; is++) {
      int A[4] = {0, 0, 0, 0}, B[4] = {0, 0, 0, 0}, C[4] = {0, 0, 0, 0};
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const int k = 4 * is + kk;
        uint32_t L1 = ql[k], L2 = ql[8 + k], H = qh[k];
        uint32_t q[4];
        q[0] = (L1 & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
        q[1] = (L2 & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
        q[2] = ((L1 >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
        q[3] = ((L2 >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int wi = 32 * c + 8 * i + k;  // limb word of elements 128c+32i+4k..+3
          A[i] = gb_dp4a_us(q[i], xa[wi], A[i]);
          B[i] = gb_dp4a_us(q[i], xb[wi], B[i]);
          C[i] = gb_dp4a_us(q[i], xc[wi], C[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float S = (float)A[i] + (float)B[i] * kL1 + (float)C[i] * kL2;
        float sc = (float)sc8[8 * c + is + 2 * i];
        acc += sc * (xs[4 * c + i] * S - 32.f * xsum[8 * c + 2 * i + is]);
      }
    }
  }
  return d * acc;
}

// Q4_0: eight 32-element blocks per super-block, y = d*(q-8).
GB_DEV float sb_q40(const uint8_t *st, int lane, const uint32_t *xa, const uint32_t *xb,
                    const uint32_t *xc, const float *xs, const float *xsum) {
  const uint4 *u = (const uint4 *)st;
  uint4 h = u[lane];
  uint32_t dw[4] = {h.x, h.y, h.z, h.w};
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    uint4 q = u[(1 + k) * 32 + lane];
    uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    uint4 la = ((const uint4 *)xa)[2 * k], ha = ((const uint4 *)xa)[2 * k + 1];
    uint4 lb = ((const uint4 *)xb)[2 * k], hb = ((const uint4 *)xb)[2 * k + 1];
    uint4 lc = ((const uint4 *)xc)[2 * k], hc = ((const uint4 *)xc)[2 * k + 1];
    uint32_t a4[4] = {la.x, la.y, la.z, la.w}, b4[4] = {lb.x, lb.y, lb.z, lb.w},
             c4[4] = {lc.x, lc.y, lc.z, lc.w};
    uint32_t A4[4] = {ha.x, ha.y, ha.z, ha.w}, B4[4] = {hb.x, hb.y, hb.z, hb.w},
             C4[4] = {hc.x, hc.y, hc.z, hc.w};
    int Al = 0, Bl = 0, Cl = 0, Ah = 0, Bh = 0, Ch = 0;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t lo = qw[kk] & 0x0F0F0F0Fu, hi = qw[kk] & 0xF0F0F0F0u;
      Al = gb_dp4a_us(lo, a4[kk], Al);
      Bl = gb_dp4a_us(lo, b4[kk], Bl);
      Cl = gb_dp4a_us(lo, c4[kk], Cl);
      Ah = gb_dp4a_us(hi, A4[kk], Ah);
      Bh = gb_dp4a_us(hi, B4[kk], Bh);
      Ch = gb_dp4a_us(hi, C4[kk], Ch);
    }
    int A = 16 * Al + Ah, B = 16 * Bl + Bh, C = 16 * Cl + Ch;
    float S = ((float)A + (float)B * kL1 + (float)C * kL2) * 0.0625f;
    float d = gb_half_to_float((uint16_t)((dw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu));
    acc += d * (xs[k] * S - 8.f * (xsum[2 * k] + xsum[2 * k + 1]));
  }
  return acc;
}

// ---- epilogues (one warp, lane l = row 32*tile + l) -----------------------

GB_DEV uint64_t argmax_key(float v, uint32_t idx) {
  // larger value wins, then the lower index (model.Argmax, model/model.go:376)
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

struct Kp {  // kernel parameters
  GbGemvArgs a;
  int rb, nrb, stages, sbb_max;
  unsigned long long units;
};

GB_DEV void epilogue(const Kp &p, int rbk, float y0, float y1) {
  const GbGemvArgs &a = p.a;
  const GbEpiArgs &e = a.e;
  const int lane = threadIdx.x & 31;
  switch (a.epi) {
    case GB_EPI_PLAIN: {
      int r = rbk * 32 + lane;
      if (r < a.rows) e.y[r] = y0;
      break;
    }
    case GB_EPI_RESID: {
      int r = rbk * 32 + lane;
      float xn = e.x[r] + y0;  // cpu.Add, backend/cpu/cpu.go:60
      e.x[r] = xn;
      GbXPack pk{e.out_pack.a, e.out_pack.b, e.out_pack.c, e.out_pack.s, e.out_pack.sum16,
                 e.out_pack.ssq};
      gb_pack_group(pk, rbk, xn * e.wnorm[r]);
      float ss = gb_warp_sum(xn * xn);
      if (lane == 0) pk.ssq[rbk] = ss;
      break;
    }
    case GB_EPI_SWIGLU: {  // cpu.SiluMul, backend/cpu/cpu.go:53
      float g = y0, u = y1;
      float ex = (float)exp(-(double)g);
      float act = g / (1.f + ex) * u;
      GbXPack pk{e.out_pack.a, e.out_pack.b, e.out_pack.c, e.out_pack.s, e.out_pack.sum16,
                 nullptr};
      gb_pack_group(pk, rbk, act);
      break;
    }
    case GB_EPI_QKV: {
      int r = rbk * 32 + lane;
      int pos = *e.pos;
      bool ok = pos >= 0 && pos < e.max_len;
      if (!ok) {
        if (lane == 0 && e.err) atomicOr(e.err, GB_DEVERR_POS);
        break;
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
        size_t idx = ((size_t)h * e.max_len + pos) * hd + dd;
        if (e.kv_f16)
          ((uint16_t *)e.vcache)[idx] = gb_float_to_half_rn(out);
        else
          ((float *)e.vcache)[idx] = out;
      }
      break;
    }
    case GB_EPI_LOGITS: {
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
        unsigned long long *best = e.best;
        atomicMax(best, (unsigned long long)key);
        __threadfence();
        unsigned done = atomicAdd(e.counter, 1u);
        if (done + 1 == (unsigned)p.nrb) {
          __threadfence();
          unsigned long long k = atomicAdd(best, 0ull);
          int32_t tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
          if (e.token_out) *e.token_out = tok;
          if (e.key_out) *e.key_out = k;  // tensor parallel: reduced across ranks next
          if (e.token_hist) {
            int pos = *e.pos;
            if (pos >= 0 && pos < e.max_len) e.token_hist[pos] = tok;
          }
          *best = 0ull;
          *e.counter = 0u;
        }
      }
      break;
    }
  }
}

// Warp `w` of the grid owns units [U*w/Wt, U*(w+1)/Wt).
GB_DEV unsigned long long unit_begin(unsigned long long U, unsigned long long Wt,
                                     unsigned long long w) {
  return U * w / Wt;
}

// Warp (of Wt) whose range contains unit u.
GB_DEV unsigned long long warp_of_unit(unsigned long long U, unsigned long long Wt,
                                       unsigned long long u) {
  unsigned long long w = (u * Wt) / U;
  while (w > 0 && unit_begin(U, Wt, w) > u) w--;
  while (w + 1 < Wt && unit_begin(U, Wt, w + 1) <= u) w++;
  return w;
}

__global__ void __launch_bounds__(512) gemv_kernel(const Kp p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GbGemvArgs &a = p.a;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int rb = p.rb, nsb = a.nsb, stages = p.stages, sbb_max = p.sbb_max;
  const unsigned long long U = p.units, Wt = (unsigned long long)gridDim.x * W;
  const unsigned long long gw = (unsigned long long)blockIdx.x * W + warp;
  const unsigned long long u0 = unit_begin(U, Wt, gw), u1 = unit_begin(U, Wt, gw + 1);
  const int n = (int)(u1 - u0);

  // shared memory: [stages rings][mbarriers][x pack planes][x scales][x sums][reduce]
  uint8_t *ring = smem + (size_t)warp * stages * rb * sbb_max;
  uint64_t *bars = (uint64_t *)(smem + (size_t)W * stages * rb * sbb_max) + warp * stages;
  const int K = nsb * 256;
  // barrier region rounded to 128 bytes: the pack planes below take 16-byte vector accesses
  uint8_t *xbase = smem + (size_t)W * stages * rb * sbb_max + (((size_t)W * stages * 8 + 127) & ~(size_t)127);
  uint32_t *xa_s = (uint32_t *)xbase;
  uint32_t *xb_s = xa_s + K / 4;
  uint32_t *xc_s = xb_s + K / 4;
  float *xs_s = (float *)(xc_s + K / 4);
  float *xsum_s = xs_s + K / 32;
  float *misc = xsum_s + K / 16;  // [0] = RMSNorm inverse

  const size_t sbb_a = (size_t)gb_tiled_sb_bytes(a.type_a), sbb_b = (size_t)gb_tiled_sb_bytes(a.type_b);
  auto tile_type = [&](int tile) { return tile < a.split_tile ? a.type_a : a.type_b; };
  auto tile_ptr = [&](int tile, int sb) -> const uint8_t * {
    if (tile < a.split_tile) return a.w + ((size_t)tile * nsb + sb) * sbb_a;
    return a.w + (size_t)a.split_tile * nsb * sbb_a + ((size_t)(tile - a.split_tile) * nsb + sb) * sbb_b;
  };
  auto issue = [&](int i) {  // bring unit u0+i into ring slot i % stages (lane 0 only)
    unsigned long long u = u0 + i;
    int rbk = (int)(u / nsb), sb = (int)(u % nsb), s = i % stages;
    uint32_t bytes = 0;
    for (int t = 0; t < rb; t++) bytes += (uint32_t)gb_tiled_sb_bytes(tile_type(rbk * rb + t));
    gb_mbar_expect_tx(&bars[s], bytes);
    for (int t = 0; t < rb; t++) {
      int tile = rbk * rb + t;
      gb_bulk_g2s(ring + ((size_t)s * rb + t) * sbb_max, tile_ptr(tile, sb),
                  (uint32_t)gb_tiled_sb_bytes(tile_type(tile)), &bars[s]);
    }
  };

  // 1. weights do not depend on the previous kernel: start their copies first
  if (lane == 0) {
    for (int s = 0; s < stages; s++) gb_mbar_init(&bars[s], 1);
    gb_mbar_fence_init();
  }
  __syncwarp();
  if (lane == 0)
    for (int i = 0; i < n && i < stages; i++) issue(i);

  // 2. the activation pack is produced by the preceding kernel
  gb_grid_dep_wait();
  {
    // RMSNorm inverse from the per-group sums of squares (cpu.RMSNorm,
    // backend/cpu/cpu.go:17: inv = 1/sqrt(sum/n + eps) in float64)
    if (a.in_ssq) {
      __shared__ double red[16];
      double ss = 0;
      for (int g = threadIdx.x; g < K / 32; g += blockDim.x) ss += (double)a.in_ssq[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        double t = 0;
        for (int w2 = 0; w2 < W; w2++) t += red[w2];
        misc[0] = (float)(1.0 / sqrt(t / (double)K + (double)a.eps));
      }
      __syncthreads();
    }
    const float inv = a.in_ssq ? misc[0] : 1.f;
    // Stage the pack for the super-blocks this CTA touches.
    const unsigned long long cu0 = unit_begin(U, Wt, (unsigned long long)blockIdx.x * W);
    const unsigned long long cu1 = unit_begin(U, Wt, (unsigned long long)(blockIdx.x + 1) * W);
    int nsbs = (cu1 - cu0) >= (unsigned long long)nsb ? nsb : (int)(cu1 - cu0);
    int sbf = (int)(cu0 % nsb);
    for (int i = threadIdx.x; i < nsbs * 16 * 3; i += blockDim.x) {
      int plane = i / (nsbs * 16), rest = i % (nsbs * 16);
      int sb = (sbf + rest / 16) % nsb, v = rest % 16;
      const int8_t *src = plane == 0 ? a.in.a : plane == 1 ? a.in.b : a.in.c;
      uint32_t *dst = plane == 0 ? xa_s : plane == 1 ? xb_s : xc_s;
      ((uint4 *)(dst + sb * 64))[v] = __ldcg((const uint4 *)(src + sb * 256) + v);
    }
    for (int i = threadIdx.x; i < nsbs * 24; i += blockDim.x) {
      int sb = (sbf + i / 24) % nsb, v = i % 24;
      if (v < 8)
        xs_s[sb * 8 + v] = __ldcg(a.in.s + sb * 8 + v) * inv;
      else
        xsum_s[sb * 16 + v - 8] = __ldcg(a.in.sum16 + sb * 16 + v - 8) * inv;
    }
  }
  __syncthreads();
  gb_grid_dep_launch();

  // 3. stream the units
  float acc0 = 0.f, acc1 = 0.f;
  bool timeout = false;
  int cur = n > 0 ? (int)(u0 / nsb) : 0;
  unsigned long long seg = u0;
  auto flush = [&](int rbk, unsigned long long s_begin, unsigned long long s_end) {
    const unsigned long long R0 = (unsigned long long)rbk * nsb, R1 = R0 + nsb;
    if (s_begin == R0 && s_end == R1) {
      epilogue(p, rbk, acc0, acc1);
      return;
    }
    const int which = u0 >= R0 ? 0 : 1;
    float *slot = a.e.part + (gw * 2 + which) * 64;
    slot[lane] = acc0;
    slot[32 + lane] = acc1;
    __threadfence();
    __syncwarp();
    unsigned done = 0;
    if (lane == 0) done = atomicAdd(a.e.tile_counter + rbk, (unsigned)(s_end - s_begin)) + (unsigned)(s_end - s_begin);
    done = __shfl_sync(0xffffffffu, done, 0);
    if (done != (unsigned)nsb) return;
    __threadfence();
    const unsigned long long wf = warp_of_unit(U, Wt, R0), wl = warp_of_unit(U, Wt, R1 - 1);
    float y0 = 0.f, y1 = 0.f;
    for (unsigned long long w2 = wf; w2 <= wl; w2++) {
      unsigned long long b2 = unit_begin(U, Wt, w2), e2 = unit_begin(U, Wt, w2 + 1);
      if (b2 == e2) continue;
      const float *sl = a.e.part + (w2 * 2 + (b2 >= R0 ? 0 : 1)) * 64;
      y0 += __ldcg(sl + lane);
      y1 += __ldcg(sl + 32 + lane);
    }
    if (lane == 0) a.e.tile_counter[rbk] = 0u;
    epilogue(p, rbk, y0, y1);
  };

  int issued = n < stages ? n : stages;
  int i = 0;
  for (; i < n; i++) {
    const unsigned long long u = u0 + i;
    const int rbk = (int)(u / nsb), sb = (int)(u % nsb), s = i % stages;
    if (rbk != cur) {
      flush(cur, seg, u);
      acc0 = acc1 = 0.f;
      cur = rbk;
      seg = u;
    }
    if (!gb_mbar_wait(&bars[s], (uint32_t)((i / stages) & 1))) {
      timeout = true;
      break;
    }
    const uint32_t *xa = xa_s + sb * 64, *xb = xb_s + sb * 64, *xc = xc_s + sb * 64;
    const float *xs = xs_s + sb * 8, *xsum = xsum_s + sb * 16;
#pragma unroll 1
    for (int t = 0; t < rb; t++) {
      const uint8_t *st = ring + ((size_t)s * rb + t) * sbb_max;
      int ty = tile_type(rbk * rb + t);
      float v = ty == GB_T_Q4_K ? sb_q4k(st, lane, xa, xb, xc, xs, xsum)
              : ty == GB_T_Q6_K ? sb_q6k(st, lane, xa, xb, xc, xs, xsum)
                                : sb_q40(st, lane, xa, xb, xc, xs, xsum);
      if (t == 0) acc0 += v; else acc1 += v;
    }
    __syncwarp();
    if (i + stages < n) {
      if (lane == 0) {
        gb_fence_proxy_async();
        issue(i + stages);
      }
      issued++;
    }
  }
  if (timeout) {
    if (lane == 0 && a.e.err) atomicOr(a.e.err, GB_DEVERR_TIMEOUT);
    // let the copies still in flight land (bounded) before the CTA exits
    for (int j = i + 1; j < issued; j++) (void)gb_mbar_wait(&bars[j % stages], (uint32_t)((j / stages) & 1));
    return;
  }
  if (n > 0) flush(cur, seg, u1);
}

// ---- repack raw ggml rows into the tiled layout (load time) ---------------
__global__ void repack_kernel(int typ, const uint8_t *raw, int rows, int nsb, int ntiles,
                              uint8_t *out) {
  const int units = gb_tiled_units(typ);
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
    (void)units;
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

size_t gemv_smem(int warps, int stages, int rb, int sbb_max, int K) {
  return (size_t)warps * stages * rb * sbb_max + (((size_t)warps * stages * 8 + 127) & ~(size_t)127) + 3 * (size_t)K +
         4 * (size_t)(K / 32 + K / 16) + 64;
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
  int blocks = (int)((total + 255) / 256);
  if (blocks > 65535 * 8) blocks = 65535 * 8;
  repack_kernel<<<blocks, 256, 0, st>>>(typ, raw, rows, nsb, ntiles, tiled);
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
  p.stages = p.rb == 2 ? 2 : 3;
  p.ks = 1;
  (void)ntiles;
  (void)nsb;
  (void)nsm;
  return p;
}

int gb_gemv_scratch_floats(int ntiles, const GbGemvPlan &p) {
  (void)ntiles;
  // two 64-float partial slots per warp of the persistent grid
  return sms() * 2 * p.warps * 2 * 64;
}

int gb_gemv_launch(const GbGemvArgs &a, const GbGemvPlan &plan, cudaStream_t st, bool pdl) {
  if (a.nsb <= 0 || a.ntiles <= 0) return gb_fail(GB_ERR_INVALID, "gpu: gemv: empty matrix");
  Kp p;
  p.a = a;
  p.rb = plan.rb;
  if (a.ntiles % p.rb) return gb_fail(GB_ERR_INVALID, "gpu: gemv: tiles not paired");
  p.nrb = a.ntiles / p.rb;
  p.units = (unsigned long long)p.nrb * a.nsb;
  bool q6 = a.type_a == GB_T_Q6_K || (a.split_tile < a.ntiles && a.type_b == GB_T_Q6_K);
  p.sbb_max = q6 ? 6720 : 4608;
  int warps = plan.warps, stages = plan.stages;
  const int K = a.nsb * 256;
  // fit the shared memory budget (227 KB per CTA)
  size_t smem = gemv_smem(warps, stages, p.rb, p.sbb_max, K);
  while (smem > 220 * 1024 && stages > 1) smem = gemv_smem(warps, --stages, p.rb, p.sbb_max, K);
  while (smem > 220 * 1024 && warps > 1) smem = gemv_smem(--warps, stages, p.rb, p.sbb_max, K);
  if (smem > 220 * 1024) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: K=%d too large", K);
  p.stages = stages;
  int per_sm = (int)((227 * 1024) / (smem + 1024));
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 2) per_sm = 2;
  long long grid = (long long)sms() * per_sm;
  long long need = (long long)((p.units + warps - 1) / warps);
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  if (grid * warps > (long long)gb_gemv_scratch_floats(a.ntiles, plan) / 128)
    grid = gb_gemv_scratch_floats(a.ntiles, plan) / 128 / warps;
  static int smem_cap = 0;
  if (!smem_cap) {
    int dev = 0, optin = 0;
    cudaFuncAttributes fa;
    GB_CUDA(cudaGetDevice(&dev), "gpu: gemv");
    GB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "gpu: gemv");
    GB_CUDA(cudaFuncGetAttributes(&fa, gemv_kernel), "gpu: gemv");
    int cap = optin - (int)fa.sharedSizeBytes;
    GB_CUDA(cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cap),
            "gpu: gemv: shared memory attribute");
    smem_cap = cap;
  }
  if (smem > (size_t)smem_cap) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: gemv: %zu bytes of shared memory", smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)(warps * 32));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GB_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel, p), "gpu: gemv launch");
  return GB_OK;
}
