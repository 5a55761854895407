// gb_prefill.cu -- batched prefill: T prompt tokens through every layer at
// once, the reference's roadmap item "Batched prefill ... AttnPrefill" with
// its "Tensor-core GEMM for prefill: dequantize a tile of weights into
// shared memory as f16, multiply with the activation tile"
// (ROADMAP.md:36-41, 99-101; the matvec batch dimension of
// backend/gpu/gpu.go:82-86 is the API it generalises).
//
// The GEMM is a tcgen05 kernel for sm_100a. Per CTA: 128 token rows x 128
// weight rows (64 gate + 64 up rows for the fused gate/up pairs), K in stages of 64:
//  * a producer warp TMA-loads the fp16 activation tile (128-byte swizzle)
//    and bulk-copies the raw quantized bytes of the stage's weight tiles
//    (the decode path's tiled layout: per 32-row tile and super-block, a
//    block of 16-byte units, unit-major and row-minor), both on one mbarrier;
//  * dequant warps, one weight row per lane, decode the stage to binary16
//    with the bit-exact float32 element formulas (quant/quant.go:56-132) and
//    write it into shared memory in the same 128-byte-swizzled K-major
//    layout, then fence to the async proxy and arrive;
//  * one thread issues tcgen05.mma (kind::f16, M=128, N=128/256, K=16, fp32
//    accumulators in tensor memory) and commits each stage's slot back to
//    the producer through an mbarrier;
//  * after the last stage the dequant warps read the accumulators with
//    tcgen05.ld and apply the epilogue (store, residual add, SwiGLU).
// Every mbarrier wait is bounded; a timeout raises GB_DEVERR_TIMEOUT.
#include <math.h>

#include <algorithm>

#include "gb_device.cuh"
#include "gb_internal.h"

namespace {

constexpr int kBM = 128;   // token rows of a CTA (UMMA M)
constexpr int kBK = 64;    // K elements of a stage (one 128-byte swizzle row of fp16)
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxStagesTC = 8;

// ---- tcgen05 / TMA wrappers (PTX ISA 8.6+, sm_100a) ------------------------
GB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
GB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
GB_DEV void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(gb_smem_u32(dst)), "r"(ncols)
               : "memory");
}
GB_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
GB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
GB_DEV void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
GB_DEV void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(gb_smem_u32(bar))
               : "memory");
}
GB_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
GB_DEV void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          gb_smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(gb_smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile whose rows are
// 128 bytes (64 fp16) with the 128-byte swizzle; 8-row core groups 1024
// bytes apart (stride byte offset), leading byte offset unused (1), the
// sm_100 descriptor version 1, layout type 2 = SWIZZLE_128B.
GB_DEV uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulators, f16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- raw weight units ---------------------------------------------------------
// The producer stages weight bytes per tile in "raw units": for quantized
// types the tile's whole sb-block (one bulk copy covers four K-stages), for
// float types the stage's contiguous quarter of it.
GB_HD int raw_spr(int typ) { return gb_float_type(typ) ? 1 : 4; }  // K-stages per raw unit
GB_HD int raw_unit_bytes(int typ) { return gb_tiled_sb_bytes(typ) / (4 / raw_spr(typ)); }

GB_DEV uint4 lds16(const uint8_t *p) { return *(const uint4 *)p; }
GB_DEV uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *(uint32_t *)&h;
}
GB_DEV uint8_t byte_of(const uint4 &v, int i) {
  const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (uint8_t)(w >> (8 * (i & 3)));
}

// Exact small integer n (0 <= n < 2^23) as float without the conversion unit.
GB_DEV float u2f(uint32_t n) { return __fsub_rn(__uint_as_float(0x4B000000u | n), 8388608.f); }
// Byte i of w as the float 2^23 + byte (its bit pattern 0x4B0000bb).
GB_DEV float magic_byte(uint32_t w, int i) { return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + i)); }

// Q4_K scale and min of sub-block j from the 12 scale bytes (bytes 4..15 of
// the block's first unit): quant.ScaleMinQ4K, quant/quant.go:90, in registers.
GB_DEV void q4k_scale_reg(const uint4 &h, int j, uint32_t &sc, uint32_t &m) {
  if (j < 4) {
    sc = byte_of(h, 4 + j) & 63u;
    m = byte_of(h, 8 + j) & 63u;
  } else {
    const uint32_t a = byte_of(h, 8 + j), lo = byte_of(h, j), hi = byte_of(h, 4 + j);
    sc = (a & 0xFu) | ((lo >> 6) << 4);
    m = (a >> 4) | ((hi >> 6) << 4);
  }
}

// Eight values v = (b - off) * d (+ c) of the bytes of w0, w1 (b small
// integers), from their magic-number floats: one byte permute, one add and one
// multiply (or fused multiply-add) per value.
GB_DEV void bytes8_scaled(uint32_t w0, uint32_t w1, float off, float d, float c, bool fused, float *v) {
  const float k = -8388608.f - off;  // exact: 2^23 + off needs 24 bits at most
#pragma unroll
  for (int e = 0; e < 8; e++) {
    const float q = __fadd_rn(magic_byte(e < 4 ? w0 : w1, e & 3), k);
    v[e] = fused ? __fmaf_rn(d, q, c) : __fmul_rn(d, q);
  }
}

// Decode output chunk c (elements 8c..8c+7) of K-stage kc of row `lane` of
// one tile, as eight binary16 values, from the tile's whole sb-block
// (quantized types) or from the stage's piece of it (float types). The values
// are the reference's element values (quant/quant.go:44-132) in float32,
// rounded to binary16; Q4_K's (d*sc)*q - dmin*m is formed with one fused
// rounding instead of two (at most one float32 ulp apart, below the
// binary16 rounding that follows).
GB_DEV uint4 dequant_chunk(int typ, int kc, const uint8_t *raw, int lane, int c) {
  float v[8];
  switch (typ) {
    case GB_T_Q4_K: {
      const uint4 h = lds16(raw + lane * 16);
      const int hi = c >> 2, b0 = (c & 3) * 8;
      const uint4 q = lds16(raw + 512 * (1 + 2 * kc + (b0 >> 4)) + lane * 16);
      const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFF)), dmin = gb_half_to_float((uint16_t)(h.x >> 16));
      uint32_t sc, m;
      q4k_scale_reg(h, 2 * kc + hi, sc, m);
      const float ds = __fmul_rn(d, u2f(sc)), dm = __fmul_rn(dmin, u2f(m));
      uint32_t w0 = (b0 & 15) ? q.z : q.x, w1 = (b0 & 15) ? q.w : q.y;
      w0 = (hi ? w0 >> 4 : w0) & 0x0F0F0F0Fu;
      w1 = (hi ? w1 >> 4 : w1) & 0x0F0F0F0Fu;
      bytes8_scaled(w0, w1, 0.f, ds, -dm, true, v);
      break;
    }
    case GB_T_Q5_K: {  // as Q4_K with the fifth bit of each quant from qh (units 1-2)
      const uint4 h = lds16(raw + lane * 16);
      const int hi = c >> 2, b0 = (c & 3) * 8, bit = 2 * kc + hi;
      const uint4 q = lds16(raw + 512 * (3 + 2 * kc + (b0 >> 4)) + lane * 16);
      const uint4 qh = lds16(raw + 512 * (1 + (b0 >> 4)) + lane * 16);
      const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFF)), dmin = gb_half_to_float((uint16_t)(h.x >> 16));
      uint32_t sc, m;
      q4k_scale_reg(h, bit, sc, m);
      const float ds = __fmul_rn(d, u2f(sc)), dm = __fmul_rn(dmin, u2f(m));
      uint32_t w0 = (b0 & 15) ? q.z : q.x, w1 = (b0 & 15) ? q.w : q.y;
      const uint32_t h0 = (b0 & 15) ? qh.z : qh.x, h1 = (b0 & 15) ? qh.w : qh.y;
      w0 = ((hi ? w0 >> 4 : w0) & 0x0F0F0F0Fu) | (((h0 >> bit) & 0x01010101u) << 4);
      w1 = ((hi ? w1 >> 4 : w1) & 0x0F0F0F0Fu) | (((h1 >> bit) & 0x01010101u) << 4);
      bytes8_scaled(w0, w1, 0.f, ds, -dm, true, v);
      break;
    }
    case GB_T_Q4_0: {  // d*(q-8)
      const uint4 dd = lds16(raw + lane * 16);
      const int b = c >> 2, k = 2 * kc + b, cc = c & 3;
      const float d = gb_half_to_float((uint16_t)(byte_of(dd, 2 * k) | byte_of(dd, 2 * k + 1) << 8));
      const uint4 q = lds16(raw + 512 * (1 + k) + lane * 16);
      uint32_t w0 = (cc & 1) ? q.z : q.x, w1 = (cc & 1) ? q.w : q.y;
      w0 = (cc >= 2 ? w0 >> 4 : w0) & 0x0F0F0F0Fu;
      w1 = (cc >= 2 ? w1 >> 4 : w1) & 0x0F0F0F0Fu;
      bytes8_scaled(w0, w1, 8.f, d, 0.f, false, v);
      break;
    }
    case GB_T_Q8_0: {  // d*q: int8 q as the unsigned byte q+128
      const uint4 dd = lds16(raw + lane * 16);
      const int b = c >> 2, k = 2 * kc + b, u = (c >> 1) & 1, hlf = c & 1;
      const float d = gb_half_to_float((uint16_t)(byte_of(dd, 2 * k) | byte_of(dd, 2 * k + 1) << 8));
      const uint4 q = lds16(raw + 512 * (1 + 2 * k + u) + lane * 16);
      const uint32_t w0 = (hlf ? q.z : q.x) ^ 0x80808080u, w1 = (hlf ? q.w : q.y) ^ 0x80808080u;
      bytes8_scaled(w0, w1, 128.f, d, 0.f, false, v);
      break;
    }
    case GB_T_Q6_K: {  // d*sc*(q-32)
      const int cq = kc >> 1, quarter = (kc & 1) * 2 + (c >> 2), l0 = (c & 3) * 8;
      const uint8_t *ql = raw + cq * 4 * 512, *qh = raw + (8 + 2 * cq) * 512, *scp = raw + 12 * 512, *dp = raw + 13 * 512;
      const int qlb = l0 + ((quarter & 1) ? 32 : 0);
      const float d = gb_half_to_float(*(const uint16_t *)(dp + lane * 2));
      const uint4 s4 = lds16(scp + lane * 16);
      const uint4 L = lds16(ql + (qlb >> 4) * 512 + lane * 16);
      const uint4 H = lds16(qh + (l0 >> 4) * 512 + lane * 16);
      const int scv = (int)(int8_t)byte_of(s4, cq * 8 + 2 * quarter + (l0 >> 4));
      const float dsc = __fmul_rn(d, (float)scv);
      uint32_t l0w = (qlb & 15) ? L.z : L.x, l1w = (qlb & 15) ? L.w : L.y;
      uint32_t h0w = (l0 & 15) ? H.z : H.x, h1w = (l0 & 15) ? H.w : H.y;
      const int sh = 2 * quarter;
      l0w = (quarter >= 2 ? l0w >> 4 : l0w) & 0x0F0F0F0Fu;
      l1w = (quarter >= 2 ? l1w >> 4 : l1w) & 0x0F0F0F0Fu;
      const uint32_t q0 = l0w | (((h0w >> sh) & 0x03030303u) << 4), q1 = l1w | (((h1w >> sh) & 0x03030303u) << 4);
      bytes8_scaled(q0, q1, 32.f, dsc, 0.f, false, v);
      break;
    }
    case GB_T_F16:
      return lds16(raw + c * 512 + lane * 16);
    case GB_T_BF16: {
      const uint4 u = lds16(raw + c * 512 + lane * 16);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
      break;
    }
    case GB_T_F32: {
      const uint4 a = lds16(raw + (2 * c) * 512 + lane * 16), b = lds16(raw + (2 * c + 1) * 512 + lane * 16);
      v[0] = __uint_as_float(a.x), v[1] = __uint_as_float(a.y), v[2] = __uint_as_float(a.z), v[3] = __uint_as_float(a.w);
      v[4] = __uint_as_float(b.x), v[5] = __uint_as_float(b.y), v[6] = __uint_as_float(b.z), v[7] = __uint_as_float(b.w);
      break;
    }
    default:
      return make_uint4(0, 0, 0, 0);
  }
  uint4 o;
  o.x = pack_h2(v[0], v[1]);
  o.y = pack_h2(v[2], v[3]);
  o.z = pack_h2(v[4], v[5]);
  o.w = pack_h2(v[6], v[7]);
  return o;
}

struct TcArgs {
  const uint8_t *w;
  int type_a, type_b, split_tile;
  int rows, ntiles, nsb;  // weight rows (N), 32-row tiles, K / 256
  int pair;               // gate/up pairs (SWIGLU): B rows 0..127 gate, 128..255 up
  int T;                  // token rows of A
  float *y;               // PLAIN: y[T][ldy]; RESID: y[T][ldy] += acc
  int ldy;
  __half *act;            // SWIGLU: act[T][ld_act] = silu(g) * u
  int ld_act;
  int mt;                 // 128-token tiles per CTA (one TMEM accumulator each)
  int splits;             // K split over gridDim.z (> 1: fp32 partials to `part`, reduced by splitk_reduce)
  float *part;
  int nstage;             // A/B ring slots (one K-stage each)
  int rstage;             // raw ring slots (one raw unit each)
  int spr;                // K-stages per raw unit (4: quantized types, 1: float types)
  int raw_tile;           // raw bytes per tile per raw unit (max over the two types)
  int npad;               // gemm_swap_kernel: token rows padded to 16 (the MMA's N)
  unsigned *err;
};
// With F16W the weights come from the model's binary16 weight copy (the
// values dequant_chunk produces, row-major, gate/up rows grouped 64 + 64 per
// CTA) through a second tensor map, one TMA box per K-stage: no raw ring and
// no decode, the dequant warps only run the epilogue.

GB_DEV const uint8_t *sb_block(const TcArgs &g, int tile, int sb, int up, int &typ) {
  if (g.pair) {
    typ = g.type_a;
    return g.w + ((size_t)(tile * g.nsb + sb) * 2 + up) * gb_tiled_sb_bytes(typ);
  }
  if (tile < g.split_tile) {
    typ = g.type_a;
    return g.w + ((size_t)tile * g.nsb + sb) * gb_tiled_sb_bytes(typ);
  }
  typ = g.type_b;
  return g.w + (size_t)g.split_tile * g.nsb * gb_tiled_sb_bytes(g.type_a) +
         ((size_t)(tile - g.split_tile) * g.nsb + sb) * gb_tiled_sb_bytes(typ);
}

// BN: weight rows of the CTA (128: 4 tiles, or 2 gate + 2 up tiles) in NT = BN/32
// tiles. 16 dequant warps: warp w decodes tile w % NT, output chunks
// [(w / NT) * CPT, +CPT) of each row (one row per lane), so every SM
// scheduler has four decoding warps to interleave; then the producer warp,
// then the MMA warp.
constexpr int kDQ = 16;
template <int BN, int EPI, bool F16W>
__global__ void __launch_bounds__((kDQ + 3) * 32, 1)
    gemm_tc_kernel(const TcArgs g, const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b) {
  constexpr int NDQ = kDQ, NT = BN / 32, CPT = 8 * NT / NDQ;
  static_assert(NDQ % NT == 0 && CPT >= 1, "dequant split");
  constexpr int BBytes = BN * 128;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t afull[kMaxStagesTC], bfull[kMaxStagesTC], empty[kMaxStagesTC];
  __shared__ __align__(8) uint64_t rfull[kMaxStagesTC], rempty[kMaxStagesTC], accf;
  __shared__ uint32_t tmem_base;
  __shared__ int bad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = g.nstage, RS = g.rstage, SPR = g.spr, MT = g.mt;
  // this CTA's K stages [k0, k0 + nkl): whole raw units of split blockIdx.z
  const int nu = g.nsb * 4 / SPR, u0 = nu * (int)blockIdx.z / g.splits, u1 = nu * ((int)blockIdx.z + 1) / g.splits;
  const int k0 = u0 * SPR, nkl = (u1 - u0) * SPR;
  const int m0 = blockIdx.y * kBM * MT;     // first token row
  const int ABytes = kABytes * MT;          // the stage's activation tiles
  // first weight tile: 4 per CTA, or for gate/up pairs 2 of each half (B rows
  // 0..63 gate, 64..127 up; TMEM columns likewise)
  const int tile0 = blockIdx.x * (g.pair ? NT / 2 : NT);
  // [NS] A tiles | [NS] B tiles (1024-aligned) | [RS][NT] raw units
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *A0 = base, *B0 = base + (size_t)NS * ABytes, *R0 = B0 + (size_t)NS * BBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      gb_mbar_init(&afull[s], 1);
      gb_mbar_init(&bfull[s], F16W ? 1 : NDQ);
      gb_mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < RS; r++) {
      gb_mbar_init(&rfull[r], 1);
      gb_mbar_init(&rempty[r], NDQ);
    }
    gb_mbar_init(&accf, 1);
    bad = 0;
    gb_mbar_fence_init();
  }
  if (warp == NDQ + 1) {
    tmem_alloc(&tmem_base, (uint32_t)(BN * MT));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == NDQ + 2 && F16W) {
    // weight producer of the binary16 copy: per K-stage the CTA's BN weight
    // rows by TMA (128-byte swizzle, the layout the MMA reads)
    if (lane == 0) {
      int b_issued = 0;
      for (int kl = 0; kl < nkl; kl++) {
        const int s = kl % NS;
        if (kl >= NS && !gb_mbar_wait(&empty[s], ((kl / NS) - 1) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        gb_mbar_expect_tx(&bfull[s], (uint32_t)BBytes);
#pragma unroll
        for (int hb = 0; hb < BN / 128; hb++)  // 128-row boxes
          tma_load_2d(B0 + (size_t)s * BBytes + (size_t)hb * 128 * 128, &tmap_b, (k0 + kl) * kBK,
                      (int)blockIdx.x * BN + hb * 128, &bfull[s]);
        b_issued = kl + 1;
      }
      for (int j = b_issued > NS ? b_issued - NS : 0; j < b_issued; j++) (void)gb_mbar_wait(&bfull[j % NS], (j / NS) & 1);
    }
  } else if (warp == NDQ + 2) {
    // raw producer: each raw unit (the tiles' weight bytes, one bulk copy per
    // tile) as soon as its slot is free, running ahead of the activation ring
    if (lane == 0) {
      const int nr = nkl / SPR;
      int r_issued = 0;
      for (int r = 0; r < nr; r++) {
        const int rs = r % RS, k = k0 + r * SPR;
        if (r >= RS && !gb_mbar_wait(&rempty[rs], ((r / RS) - 1) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        const int sb = k >> 2, kc = k & 3;
        uint32_t bytes = 0;
        for (int j = 0; j < NT; j++) {
          const int up = g.pair && j >= 2, tile = tile0 + (g.pair ? (j & 1) : j);
          if (tile >= g.ntiles) continue;
          int typ;
          (void)sb_block(g, tile, sb, up, typ);
          bytes += (uint32_t)raw_unit_bytes(typ);
        }
        gb_mbar_expect_tx(&rfull[rs], bytes);
        for (int j = 0; j < NT; j++) {
          const int up = g.pair && j >= 2, tile = tile0 + (g.pair ? (j & 1) : j);
          if (tile >= g.ntiles) continue;
          int typ;
          const uint8_t *src = sb_block(g, tile, sb, up, typ);
          const int ub = raw_unit_bytes(typ);
          gb_bulk_g2s(R0 + ((size_t)rs * NT + j) * g.raw_tile, src + (SPR == 1 ? (size_t)kc * ub : 0), (uint32_t)ub,
                      &rfull[rs]);
        }
        r_issued = r + 1;
      }
      // copies still in flight land (bounded) before the CTA exits
      for (int j = r_issued > RS ? r_issued - RS : 0; j < r_issued; j++) (void)gb_mbar_wait(&rfull[j % RS], (j / RS) & 1);
    }
  } else if (warp == NDQ) {
    // activation producer: per K-stage the MT activation tiles by TMA
    if (lane == 0) {
      int a_issued = 0;
      for (int kl = 0; kl < nkl; kl++) {
        const int k = k0 + kl;
        const int s = kl % NS;
        if (kl >= NS && !gb_mbar_wait(&empty[s], ((kl / NS) - 1) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        gb_mbar_expect_tx(&afull[s], (uint32_t)ABytes);
        for (int mt = 0; mt < MT; mt++)
          tma_load_2d(A0 + (size_t)s * ABytes + (size_t)mt * kABytes, &tmap_a, k * kBK, m0 + mt * kBM, &afull[s]);
        a_issued = kl + 1;
      }
      for (int j = a_issued > NS ? a_issued - NS : 0; j < a_issued; j++) (void)gb_mbar_wait(&afull[j % NS], (j / NS) & 1);
    }
  } else if (warp == NDQ + 1) {
    // MMA issue: one thread
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, BN);
      for (int kl = 0; kl < nkl; kl++) {
        const int s = kl % NS;
        const uint32_t ph = (kl / NS) & 1;
        if (!gb_mbar_wait(&afull[s], ph) || !gb_mbar_wait(&bfull[s], ph)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint64_t bd = sdesc_sw128(gb_smem_u32(B0 + (size_t)s * BBytes));
        for (int mt = 0; mt < MT; mt++) {
          const uint64_t ad = sdesc_sw128(gb_smem_u32(A0 + (size_t)s * ABytes + (size_t)mt * kABytes));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++)  // K = 16 per instruction: +32 bytes in the swizzled row
            mma_f16(tmem + (uint32_t)(mt * BN), ad + 2 * kk, bd + 2 * kk, idesc, (kl | kk) != 0);
        }
        mma_commit(&empty[s]);  // the slot is free once these MMAs have read it
      }
      mma_commit(&accf);  // all issued MMAs done (also after an early stop)
    }
  } else {
    // dequant warps
    const int j = warp % NT, part = warp / NT;
    const int up = g.pair && j >= 2, tile = tile0 + (g.pair ? (j & 1) : j);
    const bool valid = tile < g.ntiles;
    const int rB = j * 32 + lane, sw = lane & 7;  // B row; its 128-byte swizzle phase
    for (int kl = 0; kl < (F16W ? 0 : nkl); kl++) {
      const int k = k0 + kl, s = kl % NS, r = kl / SPR, rs = r % RS;
      // the raw unit has landed; the B slot's previous MMAs are done
      if ((kl % SPR == 0 && !gb_mbar_wait(&rfull[rs], (r / RS) & 1)) ||
          (kl >= NS && !gb_mbar_wait(&empty[s], ((kl / NS) - 1) & 1))) {
        if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
        bad = 1;
        break;
      }
      int typ = -1;  // a tile past the matrix decodes to zeros
      if (valid) (void)sb_block(g, tile, k >> 2, up, typ);
      const uint8_t *raw = R0 + ((size_t)rs * NT + j) * g.raw_tile;
      uint8_t *row = B0 + (size_t)s * BBytes + (size_t)rB * 128;
#pragma unroll
      for (int ci = 0; ci < CPT; ci++) {
        const int c = part * CPT + ci;
        *(uint4 *)(row + ((c ^ sw) << 4)) = dequant_chunk(typ, k & 3, raw, lane, c);
      }
      gb_fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        gb_mbar_arrive(&bfull[s]);
        if (kl % SPR == SPR - 1) gb_mbar_arrive(&rempty[rs]);
      }
    }
    // epilogue: accumulators -> registers -> global. Warp w reads TMEM lanes
    // 32*(w%4).. (tcgen05.ld's rule) and a quarter of the columns.
    const bool ok = gb_mbar_wait(&accf, 0);
    tc_fence_after();
    if (!ok) {
      if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
    } else if (!bad && g.splits > 1) {
      // this split's fp32 partial of the tile: [MT*128 token rows][BN columns]
      const int quarter = warp & 3, cq = warp >> 2;
      float *pt = g.part + (((size_t)blockIdx.y * gridDim.x + blockIdx.x) * g.splits + blockIdx.z) * (size_t)(MT * kBM) * BN;
      for (int mt = 0; mt < MT; mt++) {
        const int rl = mt * kBM + quarter * 32 + lane;
        if (m0 + mt * kBM + quarter * 32 >= g.T) break;  // the reduce reads token rows < T only
        const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(mt * BN);
        for (int cc = cq * (BN / 4); cc < (cq + 1) * (BN / 4); cc += 16) {
          float v[16];
          tmem_ld16(trow + cc, v);
          if (m0 + rl >= g.T) continue;
          float *dst = pt + (size_t)rl * BN + cc;
#pragma unroll
          for (int i = 0; i < 16; i += 4) *(float4 *)(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
    } else if (!bad) {
      const int quarter = warp & 3, cq = warp >> 2;
      for (int mt = 0; mt < MT; mt++) {
      const int m = m0 + mt * kBM + quarter * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(mt * BN);
      if constexpr (EPI == GB_EPI_SWIGLU) {
        // each 128 columns: gate columns 0..63 then the up columns of the same outputs
        for (int hb = 0; hb < BN / 128; hb++) {
          const int cc = hb * 128 + cq * 16;  // gate columns cc..cc+15, up columns 64+cc..
          float gv[16], uv[16];
          tmem_ld16(trow + cc, gv);
          tmem_ld16(trow + 64 + cc, uv);
          const int n = tile0 * 32 + hb * 64 + cq * 16;
          if (m < g.T && n < g.rows) {
            uint4 o[2];
            uint32_t *ow = (uint32_t *)o;
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              float a0 = gv[i] / (1.f + (float)exp(-(double)gv[i])) * uv[i];  // cpu.SiluMul
              float a1 = gv[i + 1] / (1.f + (float)exp(-(double)gv[i + 1])) * uv[i + 1];
              ow[i / 2] = pack_h2(a0, a1);
            }
            __half *dst = g.act + (size_t)m * g.ld_act + n;
            *(uint4 *)dst = o[0];
            *(uint4 *)(dst + 8) = o[1];
          }
        }
      } else {
        for (int cc = cq * (BN / 4); cc < (cq + 1) * (BN / 4); cc += 16) {
          float v[16];
          tmem_ld16(trow + cc, v);
          const int n = tile0 * 32 + cc;
          if (m >= g.T) continue;
          float *dst = g.y + (size_t)m * g.ldy + n;
          if (n + 16 <= g.rows && (g.ldy & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              if constexpr (EPI == GB_EPI_RESID) {
                const float4 x = *(const float4 *)(dst + i);
                o.x += x.x, o.y += x.y, o.z += x.z, o.w += x.w;
              }
              *(float4 *)(dst + i) = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
              if (n + i < g.rows) dst[i] = EPI == GB_EPI_RESID ? dst[i] + v[i] : v[i];
          }
        }
      }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == NDQ + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)(BN * MT));
  }
}

// Few token rows (T <= 128) through the binary16 weight copy, with the
// operands' roles swapped so that no MMA row is wasted: the CTA's 128 weight
// rows are the MMA's M (TMEM lanes), the T token rows padded to 16 its N
// (TMEM columns), and a stage moves 16 KB of weights but only 2*NP*64 bytes
// of activations (16-row TMA boxes), so the ring holds twice the stages.
// Warps 0-3 run the epilogue (warp q reads TMEM lanes 32q..32q+31: weight
// rows), warp 4 is the TMA producer (both operands on one mbarrier), warp 5
// allocates TMEM and issues the MMAs. Gate/up pairs: lanes 0-63 hold the
// gate rows, 64-127 the up rows of the same 64 outputs; warps 2-3 hand the
// up values to warps 0-1 through shared memory (an mbarrier, bounded wait).
constexpr int kMaxStagesSW = 16;
constexpr int kSwapThreads = 6 * 32;
template <int EPI>
__global__ void __launch_bounds__(kSwapThreads) gemm_swap_kernel(const TcArgs g, const __grid_constant__ CUtensorMap tmap_a16,
                                                                 const __grid_constant__ CUtensorMap tmap_w) {
  constexpr int WB = 128 * 128;  // weight bytes of a stage
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kMaxStagesSW], empty[kMaxStagesSW], accf, xch;
  __shared__ uint32_t tmem_base;
  __shared__ int bad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = g.nstage, NP = g.npad, AB = NP * 128;  // NP: a power of two, 16..128
  const uint32_t ncols = NP < 32 ? 32u : (uint32_t)NP;
  const int nu = g.nsb * 4, u0 = nu * (int)blockIdx.z / g.splits, u1 = nu * ((int)blockIdx.z + 1) / g.splits;
  const int k0 = u0, nkl = u1 - u0;
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *W0 = base, *A0 = base + (size_t)NS * WB;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      gb_mbar_init(&full[s], 1);
      gb_mbar_init(&empty[s], 1);
    }
    gb_mbar_init(&accf, 1);
    gb_mbar_init(&xch, 2);
    bad = 0;
    gb_mbar_fence_init();
  }
  if (warp == 5) {
    tmem_alloc(&tmem_base, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  if (warp == 4) {
    if (lane == 0) {
      int issued = 0;
      for (int kl = 0; kl < nkl; kl++) {
        const int s = kl % NS, k = k0 + kl;
        if (kl >= NS && !gb_mbar_wait(&empty[s], ((kl / NS) - 1) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        gb_mbar_expect_tx(&full[s], (uint32_t)(WB + AB));
        tma_load_2d(W0 + (size_t)s * WB, &tmap_w, k * kBK, (int)blockIdx.x * 128, &full[s]);
        for (int j = 0; j < NP / 16; j++) tma_load_2d(A0 + (size_t)s * AB + j * 2048, &tmap_a16, k * kBK, 16 * j, &full[s]);
        issued = kl + 1;
      }
      for (int j = issued > NS ? issued - NS : 0; j < issued; j++) (void)gb_mbar_wait(&full[j % NS], (j / NS) & 1);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, NP);
      for (int kl = 0; kl < nkl; kl++) {
        const int s = kl % NS;
        if (!gb_mbar_wait(&full[s], (kl / NS) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint64_t ad = sdesc_sw128(gb_smem_u32(W0 + (size_t)s * WB));
        const uint64_t bd = sdesc_sw128(gb_smem_u32(A0 + (size_t)s * AB));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++) mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kl | kk) != 0);
        mma_commit(&empty[s]);
      }
      mma_commit(&accf);
    }
  } else {
    // epilogue: thread = weight row 32*warp + lane, TMEM columns = tokens
    const int row = warp * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    const bool ok = gb_mbar_wait(&accf, 0);
    tc_fence_after();
    if (!ok) {
      if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
    } else if (!bad && g.splits > 1) {
      // this split's fp32 partial: [token][128 columns], the layout splitk_reduce reads
      float *pt = g.part + ((size_t)blockIdx.x * g.splits + blockIdx.z) * (size_t)(kBM * 128);
      for (int c = 0; c < NP; c += 16) {
        float v[16];
        tmem_ld16(trow + (uint32_t)c, v);
#pragma unroll
        for (int i = 0; i < 16; i++)
          if (c + i < g.T) pt[(size_t)(c + i) * 128 + row] = v[i];
      }
    } else if (!bad) {
      if constexpr (EPI == GB_EPI_SWIGLU) {
        float *xs = (float *)base;  // [token][64] up values (the ring is idle now)
        const int n = (int)blockIdx.x * 64 + (row & 63);
        if (warp >= 2) {
          for (int c = 0; c < NP; c += 16) {
            float v[16];
            tmem_ld16(trow + (uint32_t)c, v);
#pragma unroll
            for (int i = 0; i < 16; i++)
              if (c + i < g.T) xs[(c + i) * 64 + row - 64] = v[i];
          }
          __syncwarp();
          if (lane == 0) gb_mbar_arrive(&xch);
        } else if (!gb_mbar_wait(&xch, 0)) {
          if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
        } else {
          for (int c = 0; c < NP; c += 16) {
            float gv[16];
            tmem_ld16(trow + (uint32_t)c, gv);
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int t = c + i;
              if (t < g.T && n < g.rows) {
                const float u = xs[t * 64 + row];
                g.act[(size_t)t * g.ld_act + n] = __float2half_rn(gv[i] / (1.f + (float)exp(-(double)gv[i])) * u);  // cpu.SiluMul
              }
            }
          }
        }
      } else {
        const int n = (int)blockIdx.x * 128 + row;
        for (int c = 0; c < NP; c += 16) {
          float v[16];
          tmem_ld16(trow + (uint32_t)c, v);
          if (n >= g.rows) continue;
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int t = c + i;
            if (t >= g.T) break;
            float *dst = g.y + (size_t)t * g.ldy + n;
            *dst = EPI == GB_EPI_RESID ? *dst + v[i] : v[i];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// The binary16 weight copy of one tiled matrix, row-major with K contiguous:
// element (row, col) is what dequant_chunk gives the GEMM for it, so a GEMM
// on the copy multiplies the same binary16 numbers. Rows are grouped as the
// GEMM's CTAs take them: 128 consecutive rows per CTA, for gate/up pairs 64
// gate rows then the 64 matching up rows. One CTA per (32-row tile, super-
// block[, gate/up]); thread = (K-stage of 64 columns, row).
__global__ void f16_weights_kernel(const TcArgs g, __half *w16) {
  const int t = blockIdx.x, sb = blockIdx.y, up = blockIdx.z, kc = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int typ = -1;
  const uint8_t *raw = nullptr;
  if (t < g.ntiles) {
    const uint8_t *blk = sb_block(g, t, sb, up, typ);
    raw = blk + (raw_spr(typ) == 1 ? (size_t)kc * raw_unit_bytes(typ) : 0);
  }
  const int row = g.pair ? (t >> 1) * 128 + ((t & 1) + 2 * up) * 32 + lane : t * 32 + lane;
  __half *dst = w16 + (size_t)row * ((size_t)g.nsb * 256) + (size_t)sb * 256 + kc * 64;
#pragma unroll
  for (int c = 0; c < 8; c++) *(uint4 *)(dst + c * 8) = dequant_chunk(typ, kc, raw, lane, c);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// ---- the other prefill kernels -----------------------------------------------

// Embedding rows of T tokens (quant.Row, bit-exact) into x[T][dim], and the
// tokens into the fed history at pos0 + t.
__global__ void embed_rows_kernel(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *tokens, int T,
                                  int vocab, float *x, int32_t *fed, int pos0, int max_len, unsigned *err) {
  __shared__ __align__(16) uint8_t blk[1024];
  const int sb = blockIdx.x, t = blockIdx.y;
  int tok = tokens[t];
  if (sb == 0 && threadIdx.x == 0) {
    if (fed && pos0 + t < max_len) fed[pos0 + t] = tok;
    if ((tok < 0 || tok >= vocab) && err) atomicOr(err, GB_DEVERR_TOKEN);
  }
  if (tok < 0 || tok >= vocab) tok = 0;
  const int tile = tok / 32, tl = tok % 32;
  const int sbb = gb_tiled_sb_bytes(typ), raw = gb_sb_raw_bytes(typ);
  const uint8_t *src = tiled + ((size_t)tile * nsb + sb) * sbb;
  for (int b = threadIdx.x; b < raw; b += blockDim.x) blk[b] = src[gb_tiled_offset(typ, tl, b)];
  __syncthreads();
  const int e = threadIdx.x;  // 256 threads, one element each
  float v = typ == GB_T_Q4_0   ? gb_dequant_elem(typ, blk + 18 * (e / 32), e % 32)
            : typ == GB_T_Q8_0 ? gb_dequant_elem(typ, blk + 34 * (e / 32), e % 32)
                               : gb_dequant_elem(typ, blk, e);
  x[(size_t)t * dim + sb * 256 + e] = v;
}

// RMSNorm of each row (cpu.RMSNorm, backend/cpu/cpu.go:17: float64 sum of
// squares, float32 products) to binary16: the GEMM's A operand.
// Rows whose length is a multiple of 4 (and at most kNormV * 4 * blockDim)
// keep their elements in registers between the two passes.
constexpr int kNormV = 4;
__global__ void rmsnorm_rows_f16_kernel(const float *x, const float *w, int n, float eps, __half *out) {
  const float *xr = x + (size_t)blockIdx.x * n;
  __half *o = out + (size_t)blockIdx.x * n;
  __shared__ double red[32];
  double ss = 0;
  const bool vec = (n & 3) == 0 && n <= kNormV * 4 * (int)blockDim.x && ((uintptr_t)xr & 15) == 0 &&
                   ((uintptr_t)w & 15) == 0 && ((uintptr_t)o & 7) == 0;
  float4 xv[kNormV];
  if (vec) {
#pragma unroll
    for (int j = 0; j < kNormV; j++) {
      const int i4 = threadIdx.x + j * blockDim.x;
      xv[j] = i4 < (n >> 2) ? ((const float4 *)xr)[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kNormV; j++)
      ss += (double)xv[j].x * (double)xv[j].x + (double)xv[j].y * (double)xv[j].y +
            (double)xv[j].z * (double)xv[j].z + (double)xv[j].w * (double)xv[j].w;
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * (double)xr[i];
  }
  for (int k = 16; k > 0; k >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, k);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    red[0] = t;
  }
  __syncthreads();
  const float inv = (float)(1.0 / sqrt(red[0] / (double)n + (double)eps));
  if (vec) {
#pragma unroll
    for (int j = 0; j < kNormV; j++) {
      const int i4 = threadIdx.x + j * blockDim.x;
      if (i4 >= (n >> 2)) break;
      const float4 wv = ((const float4 *)w)[i4];
      __half2 h0 = __floats2half2_rn(__fmul_rn(__fmul_rn(xv[j].x, inv), wv.x), __fmul_rn(__fmul_rn(xv[j].y, inv), wv.y));
      __half2 h1 = __floats2half2_rn(__fmul_rn(__fmul_rn(xv[j].z, inv), wv.z), __fmul_rn(__fmul_rn(xv[j].w, inv), wv.w));
      uint2 u;
      u.x = *(uint32_t *)&h0;
      u.y = *(uint32_t *)&h1;
      ((uint2 *)o)[i4] = u;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __float2half_rn(__fmul_rn(__fmul_rn(xr[i], inv), w[i]));
  }
}

// RoPE of q and k rows of every token (cpu.RoPE's float64 rotation with the
// model's angle table), q to q_out, k and v into the KV cache at pos0 + t in
// the decode path's cache layouts.
__global__ void rope_kv_kernel(const float *qkv, int ldq, int q_rows, int kv_rows, int hd, const double *rope_cs,
                               int pos0, int max_len, int kv_f16, float *q_out, void *kcache, void *vcache) {
  const int t = blockIdx.x, pos = pos0 + t;
  const float *row = qkv + (size_t)t * ldq;
  const double *cs_row = rope_cs + (size_t)pos * (hd / 2) * 2;
  const int pairs = (q_rows + kv_rows) / 2;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;  // this thread's item
  if (i < pairs + kv_rows) {
    if (i < pairs) {
      const int r = 2 * i, rr = r < q_rows ? r : r - q_rows, jj = (rr % hd) >> 1;
      const double c = cs_row[2 * jj], s = cs_row[2 * jj + 1];
      const double x0 = row[r], x1 = row[r + 1];
      const float o0 = (float)__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, s));
      const float o1 = (float)__dadd_rn(__dmul_rn(x0, s), __dmul_rn(x1, c));
      if (r < q_rows) {
        q_out[(size_t)t * q_rows + r] = o0;
        q_out[(size_t)t * q_rows + r + 1] = o1;
      } else {
        const int h = rr / hd, dd = rr % hd;
        if (kv_f16) {
          const size_t idx = (((size_t)h * (hd / 8) + dd / 8) * max_len + pos) * 8 + (dd & 7);
          ((uint16_t *)kcache)[idx] = gb_float_to_half_rn(o0);
          ((uint16_t *)kcache)[idx + 1] = gb_float_to_half_rn(o1);
        } else {
          const size_t idx = (((size_t)h * (hd / 4) + dd / 4) * max_len + pos) * 4 + (dd & 3);
          ((float *)kcache)[idx] = o0;
          ((float *)kcache)[idx + 1] = o1;
        }
      }
    } else {
      const int rr = i - pairs, h = rr / hd, dd = rr % hd;
      const float v = row[q_rows + kv_rows + rr];
      if (kv_f16) {
        const size_t idx = (((size_t)h * (hd / 8) + dd / 8) * max_len + pos) * 8 + (dd & 7);
        ((uint16_t *)vcache)[idx] = gb_float_to_half_rn(v);
      } else {
        ((float *)vcache)[((size_t)h * max_len + pos) * hd + dd] = v;
      }
    }
  }
}

// Causal attention of T query tokens (positions pos0 + t) against the cache
// (the AttnPrefill of the roadmap): one CTA per (16 tokens, KV head), the
// group's query heads, key tiles of 32 positions staged in shared memory as
// float, online softmax in float32 (the decode kernels' arithmetic).
constexpr int kPQ = 16, kPK = 32;
__global__ void __launch_bounds__(256) attn_prefill_kernel(const float *q, int T, int pos0, int n_heads, int n_kv,
                                                           int hd, const void *kcache, const void *vcache, int kv_f16,
                                                           int max_len, float scale, __half *out) {
  extern __shared__ float sm[];
  const int G = n_heads / n_kv, kvh = blockIdx.y, t0 = blockIdx.x * kPQ;
  const int HP = hd + 1;  // padded rows: lane-per-key reads hit distinct banks
  float *Ks = sm, *Vs = Ks + kPK * HP, *Qs = Vs + kPK * HP;  // Qs[kPQ*G][hd]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int R = kPQ * G;  // query rows of the CTA: row = tq * G + gi
  for (int i = threadIdx.x; i < R * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd, tq = r / G, gi = r % G;
    const int t = t0 + tq;
    Qs[i] = t < T ? q[(size_t)t * n_heads * hd + (size_t)(kvh * G + gi) * hd + d] : 0.f;
  }
  constexpr int kMaxRowsPerWarp = 16, kMaxDPerLane = 4;  // G*16/8 rows, hd/32 dims
  float mrow[kMaxRowsPerWarp], lrow[kMaxRowsPerWarp], acc[kMaxRowsPerWarp][kMaxDPerLane];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; i++) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int dd = 0; dd < kMaxDPerLane; dd++) acc[i][dd] = 0.f;
  }
  const int tmax = min(T, t0 + kPQ) - 1;
  const int kv_end = pos0 + tmax + 1;  // keys [0, kv_end)
  const int DPL = hd / 32;
  for (int kb = 0; kb < kv_end; kb += kPK) {
    __syncthreads();
    // stage K and V rows kb..kb+31 of head kvh as float
    for (int i = threadIdx.x; i < kPK * (hd / 4); i += blockDim.x) {
      const int jk = i / (hd / 4), d4 = (i % (hd / 4)) * 4, p = kb + jk;
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (p < kv_end) {
        if (kv_f16) {
          const size_t idx = (((size_t)kvh * (hd / 8) + d4 / 8) * max_len + p) * 8 + (d4 & 7);
          const uint2 kr = *(const uint2 *)((const uint16_t *)kcache + idx);
          const uint2 vr = *(const uint2 *)((const uint16_t *)vcache + idx);
          kv4 = make_float4(gb_half_to_float(kr.x & 0xFFFF), gb_half_to_float(kr.x >> 16),
                            gb_half_to_float(kr.y & 0xFFFF), gb_half_to_float(kr.y >> 16));
          vv4 = make_float4(gb_half_to_float(vr.x & 0xFFFF), gb_half_to_float(vr.x >> 16),
                            gb_half_to_float(vr.y & 0xFFFF), gb_half_to_float(vr.y >> 16));
        } else {
          kv4 = *(const float4 *)((const float *)kcache + (((size_t)kvh * (hd / 4) + d4 / 4) * max_len + p) * 4);
          vv4 = *(const float4 *)((const float *)vcache + ((size_t)kvh * max_len + p) * hd + d4);
        }
      }
      float *kr = Ks + jk * HP + d4, *vr = Vs + jk * HP + d4;
      kr[0] = kv4.x, kr[1] = kv4.y, kr[2] = kv4.z, kr[3] = kv4.w;
      vr[0] = vv4.x, vr[1] = vv4.y, vr[2] = vv4.z, vr[3] = vv4.w;
    }
    __syncthreads();
#pragma unroll
    for (int ri = 0; ri < kMaxRowsPerWarp; ri++) {
      const int r = warp + ri * nw;
      if (r >= R) break;
      const int t = t0 + r / G;
      if (t >= T) continue;
      const int qpos = pos0 + t, p = kb + lane;
      const float *qr = Qs + r * hd, *kr = Ks + lane * HP;
      float s = 0.f;
      for (int d = 0; d < hd; d++) s = fmaf(qr[d], kr[d], s);
      s = p <= qpos ? s * scale : -INFINITY;
      const float mt = gb_warp_max(s);
      const float mn = fmaxf(mrow[ri], mt);
      if (mn == -INFINITY) continue;  // no visible key in this tile yet
      const float alpha = expf(mrow[ri] - mn), pe = expf(s - mn);
      lrow[ri] = lrow[ri] * alpha + gb_warp_sum(pe);
      mrow[ri] = mn;
#pragma unroll
      for (int dd = 0; dd < kMaxDPerLane; dd++)
        if (dd < DPL) acc[ri][dd] *= alpha;
      for (int jk = 0; jk < kPK; jk++) {
        const float pj = __shfl_sync(0xffffffffu, pe, jk);
#pragma unroll
        for (int dd = 0; dd < kMaxDPerLane; dd++)
          if (dd < DPL) acc[ri][dd] = fmaf(pj, Vs[jk * HP + lane + 32 * dd], acc[ri][dd]);
      }
    }
  }
#pragma unroll
  for (int ri = 0; ri < kMaxRowsPerWarp; ri++) {
    const int r = warp + ri * nw;
    if (r >= R) break;
    const int t = t0 + r / G, gi = r % G;
    if (t >= T) continue;
    const float inv = 1.f / lrow[ri];
#pragma unroll
    for (int dd = 0; dd < kMaxDPerLane; dd++)
      if (dd < DPL)
        out[(size_t)t * n_heads * hd + (size_t)(kvh * G + gi) * hd + lane + 32 * dd] =
            __float2half_rn(acc[ri][dd] * inv);
  }
}


// Causal attention of T query tokens on the tensor cores (flash-attention
// style): one CTA per (QT tokens, KV head) with 64 query rows (token, group
// head); four warps of 16 rows; K/V tiles of 64 positions double-buffered
// in shared memory in the cache's own [16-byte dim chunk][position] order;
// S = Q K^T and O += P V with mma.sync m16n8k16. q and p are each split into
// a binary16 value and its binary16 residue (two MMAs), which keeps about 22
// bits of both, so the scores and weights carry float32-level precision and
// only the cache's binary16 K/V limit the result. Online softmax in float32.
constexpr int kFM = 64, kFK = 64;
GB_DEV void cp_async16(void *dst, const void *src, bool zero) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(gb_smem_u32(dst)), "l"(src),
               "r"(zero ? 0 : 16)
               : "memory");
}
GB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
GB_DEV void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
GB_DEV void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <bool F16, int HD>
__global__ void __launch_bounds__(128) attn_prefill_mma_kernel(const float *q, int T, int pos0, int n_heads,
                                                               int n_kv, const void *kcache, const void *vcache,
                                                               int max_len, float scale, __half *out) {
  constexpr int NC = HD / 8;                 // 16-byte chunks of a K/V row
  constexpr int TILE = NC * kFK * 8;         // halves of one K (or V) tile
  extern __shared__ __align__(128) uint16_t kvs[];  // [2 buffers][K, V][NC][kFK][8]
  const int G = n_heads / n_kv, QT = kFM / G, kvh = blockIdx.y, t0 = blockIdx.x * QT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g4 = lane >> 2, t4 = lane & 3;
  const int tlast = min(T, t0 + QT) - 1;
  const int kv_end = pos0 + tlast + 1;
  const int ntile = (kv_end + kFK - 1) / kFK;

  // this thread's two rows (g4 and g4 + 8 of the warp's 16)
  int qpos[2];
  bool rvalid[2];
  const float *qrow[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int r = warp * 16 + g4 + 8 * i, tq = r / G, gi = r % G, t = t0 + tq;
    rvalid[i] = tq < QT && t < T;
    qpos[i] = rvalid[i] ? pos0 + t : -1;
    qrow[i] = q + ((size_t)(rvalid[i] ? t : 0) * n_heads + (size_t)(kvh * G + gi)) * HD;
  }
  // Q fragments (scaled), split into binary16 value and residue
  uint32_t qh[HD / 16][4], ql[HD / 16][4];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ks++) {
#pragma unroll
    for (int half = 0; half < 2; half++)
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const int d = ks * 16 + half * 8 + 2 * t4;
        const float x0 = rvalid[i] ? qrow[i][d] * scale : 0.f, x1 = rvalid[i] ? qrow[i][d + 1] * scale : 0.f;
        split2(x0, x1, qh[ks][half * 2 + i], ql[ks][half * 2 + i]);
      }
  }

  auto stage = [&](int buf, int kb) {
    uint16_t *Kd = kvs + (size_t)buf * 2 * TILE, *Vd = Kd + TILE;
    for (int i = threadIdx.x; i < NC * kFK; i += blockDim.x) {
      const int c = i / kFK, j = i % kFK, p = kb + j;
      const bool in = p < kv_end;
      uint16_t *kd = Kd + ((size_t)c * kFK + j) * 8, *vd = Vd + ((size_t)c * kFK + j) * 8;
      if constexpr (F16) {
        const size_t off = (((size_t)kvh * NC + c) * max_len + (in ? p : 0)) * 8;
        cp_async16(kd, (const uint16_t *)kcache + off, !in);
        cp_async16(vd, (const uint16_t *)vcache + off, !in);
      } else {
        float kf[8], vf[8];
#pragma unroll
        for (int e = 0; e < 8; e++) kf[e] = vf[e] = 0.f;
        if (in) {
          const float *kb4 = (const float *)kcache;
          const float4 a = *(const float4 *)(kb4 + (((size_t)kvh * (HD / 4) + 2 * c) * max_len + p) * 4);
          const float4 b = *(const float4 *)(kb4 + (((size_t)kvh * (HD / 4) + 2 * c + 1) * max_len + p) * 4);
          const float4 va = *(const float4 *)((const float *)vcache + ((size_t)kvh * max_len + p) * HD + 8 * c);
          const float4 vb = *(const float4 *)((const float *)vcache + ((size_t)kvh * max_len + p) * HD + 8 * c + 4);
          kf[0] = a.x, kf[1] = a.y, kf[2] = a.z, kf[3] = a.w, kf[4] = b.x, kf[5] = b.y, kf[6] = b.z, kf[7] = b.w;
          vf[0] = va.x, vf[1] = va.y, vf[2] = va.z, vf[3] = va.w, vf[4] = vb.x, vf[5] = vb.y, vf[6] = vb.z, vf[7] = vb.w;
        }
        *(uint4 *)kd = make_uint4(pack_h2(kf[0], kf[1]), pack_h2(kf[2], kf[3]), pack_h2(kf[4], kf[5]), pack_h2(kf[6], kf[7]));
        *(uint4 *)vd = make_uint4(pack_h2(vf[0], vf[1]), pack_h2(vf[2], vf[3]), pack_h2(vf[4], vf[5]), pack_h2(vf[6], vf[7]));
      }
    }
    cp_async_commit();
  };

  float o[NC][4];
#pragma unroll
  for (int nd = 0; nd < NC; nd++) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  if (ntile > 0) stage(0, 0);
  for (int it = 0; it < ntile; it++) {
    const int kb = it * kFK, buf = it & 1;
    if (it + 1 < ntile) {
      stage(buf ^ 1, kb + kFK);
      cp_async_wait1();
    } else {
      cp_async_wait0();
    }
    __syncthreads();
    const uint16_t *Kt = kvs + (size_t)buf * 2 * TILE, *Vt = Kt + TILE;
    // S = Q K^T for 64 keys: 8 blocks of 8
    float sc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; nb++) sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks++)
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        const int m = lane >> 3, c = 2 * ks + (m & 1), key = 8 * (nb + (m >> 1)) + (lane & 7);
        uint32_t b[4];
        ldsm_x4(b, Kt + ((size_t)c * kFK + key) * 8);
        mma16816(sc[nb], qh[ks], b[0], b[1]);
        mma16816(sc[nb], ql[ks], b[0], b[1]);
        mma16816(sc[nb + 1], qh[ks], b[2], b[3]);
        mma16816(sc[nb + 1], ql[ks], b[2], b[3]);
      }
    // causal mask and online softmax (rows g4 and g4+8)
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int i = e >> 1, key = kb + 8 * nb + 2 * t4 + (e & 1);
        if (key > qpos[i]) sc[nb][e] = -INFINITY;
        mt[i] = fmaxf(mt[i], sc[nb][e]);
      }
    float alpha[2], base[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
      mt[i] = fmaxf(mt[i], __shfl_xor_sync(0xffffffffu, mt[i], 1));
      mt[i] = fmaxf(mt[i], __shfl_xor_sync(0xffffffffu, mt[i], 2));
      const float mn = fmaxf(mrow[i], mt[i]);
      base[i] = mn == -INFINITY ? 0.f : mn;
      alpha[i] = expf(mrow[i] - base[i]);
      mrow[i] = mn;
      lrow[i] *= alpha[i];
    }
#pragma unroll
    for (int nd = 0; nd < NC; nd++) {
      o[nd][0] *= alpha[0], o[nd][1] *= alpha[0];
      o[nd][2] *= alpha[1], o[nd][3] *= alpha[1];
    }
    // P (split) as A fragments, 16 keys per k-step
    uint32_t ph[4][4], pl[4][4];
#pragma unroll
    for (int nb = 0; nb < 8; nb++) {
      const float p0 = expf(sc[nb][0] - base[0]), p1 = expf(sc[nb][1] - base[0]);
      const float p2 = expf(sc[nb][2] - base[1]), p3 = expf(sc[nb][3] - base[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      const int kk = nb >> 1, hi = nb & 1;
      split2(p0, p1, ph[kk][hi * 2 + 0], pl[kk][hi * 2 + 0]);
      split2(p2, p3, ph[kk][hi * 2 + 1], pl[kk][hi * 2 + 1]);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; kk++)
#pragma unroll
      for (int nd = 0; nd < NC; nd += 2) {
        const int m = lane >> 3, key = 16 * kk + 8 * (m & 1) + (lane & 7), c = nd + (m >> 1);
        uint32_t b[4];
        ldsm_x4_t(b, Vt + ((size_t)c * kFK + key) * 8);
        mma16816(o[nd], ph[kk], b[0], b[1]);
        mma16816(o[nd], pl[kk], b[0], b[1]);
        mma16816(o[nd + 1], ph[kk], b[2], b[3]);
        mma16816(o[nd + 1], pl[kk], b[2], b[3]);
      }
    __syncthreads();  // the buffer is restaged two tiles later
  }
  // normalise and store
#pragma unroll
  for (int i = 0; i < 2; i++) {
    float l = lrow[i];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    lrow[i] = l > 0.f ? 1.f / l : 0.f;
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    if (!rvalid[i]) continue;
    const int r = warp * 16 + g4 + 8 * i, t = t0 + r / G, gi = r % G;
    __half *orow = out + ((size_t)t * n_heads + (size_t)(kvh * G + gi)) * HD;
#pragma unroll
    for (int nd = 0; nd < NC; nd++)
      *(uint32_t *)(orow + 8 * nd + 2 * t4) = pack_h2(o[nd][2 * i] * lrow[i], o[nd][2 * i + 1] * lrow[i]);
  }
}

// Sum of the split-K partials of gemm_tc_kernel in split order (deterministic)
// and the epilogue: PLAIN y = sum, RESID y += sum, SWIGLU act = silu(g) * u.
// One thread per 4 consecutive output columns of one token row (16-byte
// partial reads); grid (column groups, token rows).
template <int EPI>
__global__ void splitk_reduce_kernel(const float *part, int S, int MT, int BN, int ntn, int T, int rows, float *y,
                                     int ldy, __half *act, int ld_act) {
  const int m = blockIdx.y, n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (n >= rows) return;
  const size_t tile = (size_t)MT * kBM * BN;
  const int mg = m / (MT * kBM), rl = m % (MT * kBM);
  const int oc = EPI == GB_EPI_SWIGLU ? BN / 2 : BN;  // outputs of one CTA column
  // the column of output n in its CTA's tile (gate/up: per 128 columns, 64 gate then 64 up)
  const int col = EPI == GB_EPI_SWIGLU ? (n % oc) / 64 * 128 + n % 64 : n % oc;
  const float *p = part + ((size_t)mg * ntn + n / oc) * S * tile + (size_t)rl * BN + col;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = v;
  for (int z = 0; z < S; z++) {
    const float4 a = __ldcg((const float4 *)(p + z * tile));
    v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
    if constexpr (EPI == GB_EPI_SWIGLU) {
      const float4 b = __ldcg((const float4 *)(p + z * tile + 64));
      u.x += b.x, u.y += b.y, u.z += b.z, u.w += b.w;
    }
  }
  const float vv[4] = {v.x, v.y, v.z, v.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    if (n + i >= rows) break;
    if constexpr (EPI == GB_EPI_SWIGLU) {
      act[(size_t)m * ld_act + n + i] = __float2half_rn(vv[i] / (1.f + (float)exp(-(double)vv[i])) * uu[i]);  // cpu.SiluMul
    } else if constexpr (EPI == GB_EPI_RESID) {
      y[(size_t)m * ldy + n + i] += vv[i];
    } else {
      y[(size_t)m * ldy + n + i] = vv[i];
    }
  }
}

}  // namespace

// ---- launchers ------------------------------------------------------------------

int gb_tmap_f16_rows(const void *base, int rows, int cols, CUtensorMap *map, int box_rows) {
  static EncodeTiledFn encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return gb_fail(GB_ERR_CUDA, "gpu: prefill: cuTensorMapEncodeTiled unavailable");
    encode = (EncodeTiledFn)fn;
  }
  if (cols % kBK || ((uintptr_t)base & 15)) return gb_fail(GB_ERR_INVALID, "gpu: prefill: bad activation layout");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return gb_fail(GB_ERR_CUDA, "gpu: prefill: tensor map encode failed (%d)", (int)r);
  return GB_OK;
}

// Token tiles per CTA (MT: one weight decode feeds MT MMAs; at most 512 TMEM
// columns) and K splits (S: enough CTAs for one wave over the SMs when the
// weight tiles alone are too few; whole raw units per split).
GbTcPlan gb_tc_gemm_plan(const GbTcGemm &a, int sms) {
  GbTcPlan p;
  const bool pair = a.epi == GB_EPI_SWIGLU;
  if (a.w16 && a.a16 && a.T <= kBM) {
    // gemm_swap_kernel: K splits for about two CTAs per SM, each split at
    // least four K-stages long
    const int ntn = (a.rows + (pair ? 63 : 127)) / (pair ? 64 : 128), nu = a.nsb * 4;
    int S = (2 * sms) / std::max(1, ntn);
    S = std::max(1, std::min(S, nu / 4));
    p.swap = true;
    p.splits = S;
    p.part_floats = S > 1 ? (size_t)ntn * S * kBM * 128 : 0;
    return p;
  }
  // with the binary16 copy: 256 weight rows and up to 2 token tiles per CTA
  // (a stage of 32 KB activations + 32 KB weights, three stages), else 128 rows
  // and up to 4 token tiles (the dequant warps' width)
  const bool wide = a.w16 != nullptr;
  const int BN = wide ? 256 : 128, mt_max = wide ? 2 : 4, oc = pair ? BN / 2 : BN;
  const int mtiles = (a.T + kBM - 1) / kBM, ntn = (a.rows + oc - 1) / oc;
  int mt = 1;
  while (mt * 2 <= mt_max && mt * 2 <= mtiles) mt *= 2;
  const int mg = (mtiles + mt - 1) / mt;
  const int spr = gb_float_type(a.type_a) ? 1 : 4, nu = a.nsb * 4 / spr;
  int S = sms / std::max(1, ntn * mg);
  S = std::max(1, std::min(S, std::min(nu, 8)));
  p.mt = mt;
  p.splits = S;
  p.part_floats = S > 1 ? (size_t)ntn * mg * S * mt * kBM * BN : 0;
  return p;
}

int gb_tc_gemm_launch(const GbTcGemm &a, cudaStream_t st) {
  if (a.T <= 0) return GB_OK;
  if (a.nsb <= 0 || (a.epi == GB_EPI_SWIGLU && (a.rows % 16 || a.ld_act % 8)))
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: %d rows, %d super-blocks", a.rows, a.nsb);
  if (!gb_tiled_type(a.type_a) || !gb_tiled_type(a.type_b))
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: weight type %d/%d", a.type_a, a.type_b);
  TcArgs g{};
  g.w = a.w;
  g.type_a = a.type_a;
  g.type_b = a.type_b;
  g.split_tile = a.split_tile;
  g.rows = a.rows;
  g.ntiles = a.ntiles;
  g.nsb = a.nsb;
  g.pair = a.epi == GB_EPI_SWIGLU;
  g.T = a.T;
  g.y = a.y;
  g.ldy = a.ldy;
  g.act = a.act;
  g.ld_act = a.ld_act;
  g.err = a.err;
  g.spr = std::min(raw_spr(a.type_a), raw_spr(a.type_b));
  if (raw_spr(a.type_a) != raw_spr(a.type_b))
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: mixed quantized and float tiles");
  g.raw_tile = (std::max(raw_unit_bytes(a.type_a), raw_unit_bytes(a.type_b)) + 127) & ~127;
  const bool f16w = a.w16 != nullptr;
  const int BN = f16w ? 256 : 128, NT = BN / 32, oc = g.pair ? BN / 2 : BN;
  const int mtiles = (a.T + kBM - 1) / kBM, ntn = (a.rows + oc - 1) / oc;
  GbTcPlan plan = gb_tc_gemm_plan(a, 148);
  if (plan.splits > 1 && (!a.part || a.part_floats < plan.part_floats)) {  // no room for partials: one split
    plan.splits = 1;
    plan.part_floats = 0;
  }
  const int mt = plan.mt;
  g.splits = plan.splits;
  g.part = a.part;
  g.mt = mt;
  int rbn = BN, rntn = ntn;  // the partials' tile width and CTA columns, for the reduce
  if (plan.swap) {
    int np = 16;
    while (np < a.T) np *= 2;
    g.npad = np;
    const int sw_ntn = (a.rows + (g.pair ? 63 : 127)) / (g.pair ? 64 : 128);  // 128 weight rows per CTA
    const int nctas = sw_ntn * g.splits;
    rbn = 128;
    rntn = sw_ntn;
    const int resident = std::max(1, std::min(4, (nctas + 147) / 148));  // CTAs an SM holds at once
    const size_t per_cta = (size_t)233472 / resident - 2048 - 1024;  // minus reserved/static and alignment slack
    const size_t stage = (size_t)128 * 128 + (size_t)np * 128;
    const int ns = (int)std::min<size_t>(kMaxStagesSW, per_cta / stage);
    if (ns < 2) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: stages do not fit");
    g.nstage = ns;
    const size_t smem = (size_t)ns * stage + 1024;
    void (*kern)(TcArgs, CUtensorMap, CUtensorMap) =
        a.epi == GB_EPI_PLAIN ? gemm_swap_kernel<GB_EPI_PLAIN>
                              : a.epi == GB_EPI_RESID ? gemm_swap_kernel<GB_EPI_RESID> : gemm_swap_kernel<GB_EPI_SWIGLU>;
    GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "gpu: GEMM");
    kern<<<dim3((unsigned)sw_ntn, 1, (unsigned)g.splits), kSwapThreads, smem, st>>>(g, a.tmap_a16, a.tmap_b);
    GB_CUDA(cudaGetLastError(), "gpu: GEMM");
  } else {
  const size_t ab = (size_t)kABytes * mt + (size_t)BN * 128, rb = (size_t)NT * g.raw_tile;
  const size_t budget = 227 * 1024 - 1024 - 512;  // dynamic smem minus the alignment slack and statics
  // (A/B slots, raw slots) in order of preference: two raw units in flight
  // keep the copy of the next super-block under the decode of this one
  static const int pref[9][2] = {{4, 3}, {4, 2}, {3, 3}, {3, 2}, {2, 3}, {2, 2}, {4, 1}, {3, 1}, {2, 1}};
  int ns = 0, rsn = 0;
  if (f16w) {  // binary16 weights by TMA: every byte of shared memory to the A/B ring
    ns = (int)std::min<size_t>(kMaxStagesTC, budget / ab);
    if (ns < 2) ns = 0;
  } else {
    for (const auto &p : pref)
      if (p[0] * ab + p[1] * rb <= budget) {
        ns = p[0];
        rsn = p[1];
        break;
      }
  }
  if (!ns) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: stages do not fit");
  g.nstage = ns;
  g.rstage = rsn;
  const size_t stage = ab;
  const size_t smem = (size_t)ns * stage + (size_t)rsn * rb + 1024;
  const dim3 grid((unsigned)ntn, (unsigned)((mtiles + mt - 1) / mt), (unsigned)g.splits);
  const dim3 block((unsigned)((kDQ + 3) * 32));
  void (*kern)(TcArgs, CUtensorMap, CUtensorMap) = nullptr;
  switch (a.epi) {
    case GB_EPI_PLAIN:
      kern = f16w ? gemm_tc_kernel<256, GB_EPI_PLAIN, true> : gemm_tc_kernel<128, GB_EPI_PLAIN, false>;
      break;
    case GB_EPI_RESID:
      kern = f16w ? gemm_tc_kernel<256, GB_EPI_RESID, true> : gemm_tc_kernel<128, GB_EPI_RESID, false>;
      break;
    case GB_EPI_SWIGLU:
      kern = f16w ? gemm_tc_kernel<256, GB_EPI_SWIGLU, true> : gemm_tc_kernel<128, GB_EPI_SWIGLU, false>;
      break;
    default: return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: epilogue %d", a.epi);
  }
  GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "gpu: prefill GEMM");
  kern<<<grid, block, smem, st>>>(g, a.tmap_a, f16w ? a.tmap_b : a.tmap_a);
  GB_CUDA(cudaGetLastError(), "gpu: prefill GEMM");
  }
  if (g.splits > 1) {
    const dim3 blocks((unsigned)((a.rows + 4 * 128 - 1) / (4 * 128)), (unsigned)a.T);
    switch (a.epi) {
      case GB_EPI_PLAIN:
        splitk_reduce_kernel<GB_EPI_PLAIN><<<blocks, 128, 0, st>>>(a.part, g.splits, mt, rbn, rntn, a.T, a.rows, a.y,
                                                                   a.ldy, nullptr, 0);
        break;
      case GB_EPI_RESID:
        splitk_reduce_kernel<GB_EPI_RESID><<<blocks, 128, 0, st>>>(a.part, g.splits, mt, rbn, rntn, a.T, a.rows, a.y,
                                                                   a.ldy, nullptr, 0);
        break;
      default:
        splitk_reduce_kernel<GB_EPI_SWIGLU><<<blocks, 128, 0, st>>>(a.part, g.splits, mt, rbn, rntn, a.T, a.rows,
                                                                    nullptr, 0, a.act, a.ld_act);
    }
    GB_CUDA(cudaGetLastError(), "gpu: prefill split-K reduce");
  }
  return GB_OK;
}

// Rows of the binary16 weight copy of a GEMM's matrix: 128 per CTA column.
size_t gb_tc_f16_rows(const GbTcGemm &a) {
  const bool pair = a.epi == GB_EPI_SWIGLU;
  return (size_t)((a.rows + (pair ? 63 : 127)) / (pair ? 64 : 128)) * 128;
}

int gb_tc_f16_weights_launch(const GbTcGemm &a, __half *w16, CUtensorMap *map, cudaStream_t st) {
  if (a.nsb <= 0 || !gb_tiled_type(a.type_a) || !gb_tiled_type(a.type_b) || ((uintptr_t)w16 & 15))
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: binary16 weights: type %d/%d, %d super-blocks", a.type_a, a.type_b,
                   a.nsb);
  TcArgs g{};
  g.w = a.w;
  g.type_a = a.type_a;
  g.type_b = a.type_b;
  g.split_tile = a.split_tile;
  g.rows = a.rows;
  g.ntiles = a.ntiles;
  g.nsb = a.nsb;
  g.pair = a.epi == GB_EPI_SWIGLU;
  const size_t rows16 = gb_tc_f16_rows(a);
  const dim3 grid((unsigned)(rows16 / (g.pair ? 64 : 32)), (unsigned)a.nsb, g.pair ? 2u : 1u);  // (tile, sb, up)
  f16_weights_kernel<<<grid, 128, 0, st>>>(g, w16);
  GB_CUDA(cudaGetLastError(), "gpu: binary16 weights");
  return gb_tmap_f16_rows(w16, (int)rows16, a.nsb * 256, map);
}

int gb_embed_rows_launch(int typ, const uint8_t *tiled, int nsb, int dim, const int32_t *tokens, int T, int vocab,
                         float *x, int32_t *fed, int pos0, int max_len, unsigned *err, cudaStream_t st) {
  embed_rows_kernel<<<dim3((unsigned)(dim / 256), (unsigned)T), 256, 0, st>>>(typ, tiled, nsb, dim, tokens, T, vocab,
                                                                                x, fed, pos0, max_len, err);
  GB_CUDA(cudaGetLastError(), "gpu: prefill embedding");
  return GB_OK;
}

int gb_rmsnorm_rows_f16_launch(const float *x, const float *w, int rows, int n, float eps, __half *out,
                               cudaStream_t st) {
  rmsnorm_rows_f16_kernel<<<rows, 512, 0, st>>>(x, w, n, eps, out);
  GB_CUDA(cudaGetLastError(), "gpu: prefill RMSNorm");
  return GB_OK;
}

int gb_rope_kv_launch(const float *qkv, int T, int q_rows, int kv_rows, int hd, const double *rope_cs, int pos0,
                      int max_len, int kv_f16, float *q_out, void *kcache, void *vcache, cudaStream_t st) {
  const unsigned items = (unsigned)((q_rows + kv_rows) / 2 + kv_rows);
  rope_kv_kernel<<<dim3((unsigned)T, (items + 255) / 256), 256, 0, st>>>(qkv, q_rows + 2 * kv_rows, q_rows, kv_rows, hd, rope_cs, pos0, max_len, kv_f16,
                                    q_out, kcache, vcache);
  GB_CUDA(cudaGetLastError(), "gpu: prefill RoPE");
  return GB_OK;
}

int gb_attn_prefill_launch(const float *q, int T, int pos0, int n_heads, int n_kv, int hd, const void *kcache,
                           const void *vcache, int kv_f16, int max_len, __half *out, cudaStream_t st) {
  const int G = n_heads / n_kv;
  if ((hd == 64 || hd == 128) && G <= kFM) {
    // tensor-core path
    const int QT = kFM / G;
    const size_t smem = (size_t)2 * 2 * (hd / 8) * kFK * 16;
    void (*kern)(const float *, int, int, int, int, const void *, const void *, int, float, __half *) =
        hd == 64 ? (kv_f16 ? attn_prefill_mma_kernel<true, 64> : attn_prefill_mma_kernel<false, 64>)
                 : (kv_f16 ? attn_prefill_mma_kernel<true, 128> : attn_prefill_mma_kernel<false, 128>);
    GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
            "gpu: prefill attention");
    kern<<<dim3((unsigned)((T + QT - 1) / QT), (unsigned)n_kv), 128, smem, st>>>(
        q, T, pos0, n_heads, n_kv, kcache, vcache, max_len, 1.f / sqrtf((float)hd), out);
    GB_CUDA(cudaGetLastError(), "gpu: prefill attention");
    return GB_OK;
  }
  if (hd % 32 || hd > 128 || G * kPQ > 16 * 8)
    return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill attention: head_dim %d, group %d", hd, G);
  const size_t smem = sizeof(float) * ((size_t)2 * kPK * (hd + 1) + (size_t)kPQ * G * hd);
  GB_CUDA(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "gpu: prefill attention");
  attn_prefill_kernel<<<dim3((unsigned)((T + kPQ - 1) / kPQ), (unsigned)n_kv), 256, smem, st>>>(
      q, T, pos0, n_heads, n_kv, hd, kcache, vcache, kv_f16, max_len, 1.f / sqrtf((float)hd), out);
  GB_CUDA(cudaGetLastError(), "gpu: prefill attention");
  return GB_OK;
}
