// gb_prefill.cu -- batched prefill: T prompt tokens through every layer at
// once, the reference's roadmap item "Batched prefill ... AttnPrefill" with
// its "Tensor-core GEMM for prefill: dequantize a tile of weights into
// shared memory as f16, multiply with the activation tile"
// (ROADMAP.md:36-41, 99-101; the matvec batch dimension of
// backend/gpu/gpu.go:82-86 is the API it generalises).
//
// The GEMM is a tcgen05 kernel for sm_100a. Per CTA: 128 token rows x 128
// weight rows (256 for the fused gate/up pairs), K in stages of 64:
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

// ---- one stage of weight bytes per tile -----------------------------------
// The 16-byte units of a super-block that K-stage kc (elements 64kc..64kc+63)
// needs, as (byte offset in the sb-block, bytes) pieces; packed in this
// order in the stage's raw region of the tile.
struct Piece {
  int off, len;
};
GB_HD int stage_pieces(int typ, int kc, Piece *pc) {
  switch (typ) {
    case GB_T_Q4_K:
    case GB_T_Q4_0:
      pc[0] = {0, 512};
      pc[1] = {(1 + 2 * kc) * 512, 1024};
      return 2;
    case GB_T_Q8_0:
      pc[0] = {0, 512};
      pc[1] = {(1 + 4 * kc) * 512, 2048};
      return 2;
    case GB_T_Q6_K: {
      const int c = kc >> 1;
      pc[0] = {c * 4 * 512, 2048};        // ql bytes 64c..64c+63
      pc[1] = {(8 + 2 * c) * 512, 1024};  // qh bytes 32c..32c+31
      pc[2] = {12 * 512, 512};            // the 16 int8 scales
      pc[3] = {13 * 512, 64};             // d of the 32 rows
      return 4;
    }
    case GB_T_F16:
    case GB_T_BF16:
      pc[0] = {8 * kc * 512, 4096};
      return 1;
    case GB_T_F32:
      pc[0] = {16 * kc * 512, 8192};
      return 1;
  }
  return 0;
}
GB_HD int stage_raw_bytes(int typ) {
  Piece pc[4];
  int n = stage_pieces(typ, 0, pc), b = 0;
  for (int i = 0; i < n; i++) b += pc[i].len;
  return b;
}

GB_DEV uint4 lds16(const uint8_t *p) { return *(const uint4 *)p; }
GB_DEV uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *(uint32_t *)&h;
}
GB_DEV uint8_t byte_of(const uint4 &v, int i) {
  const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (uint8_t)(w >> (8 * (i & 3)));
}

// Decode K-stage kc of row `lane` of one tile from its raw stage bytes into
// the fp16 B tile row rB (swizzled). Values are the reference's float32
// element values rounded to binary16.
GB_DEV void dequant_stage(int typ, int kc, const uint8_t *raw, int lane, uint8_t *btile, int rB) {
  uint8_t *row = btile + rB * 128;
  const int sw = rB & 7;
  auto put = [&](int c, const float *v) {
    uint4 o;
    o.x = pack_h2(v[0], v[1]);
    o.y = pack_h2(v[2], v[3]);
    o.z = pack_h2(v[4], v[5]);
    o.w = pack_h2(v[6], v[7]);
    *(uint4 *)(row + ((c ^ sw) << 4)) = o;
  };
  float v[8];
  switch (typ) {
    case GB_T_Q4_K: {  // quant/quant.go:97-112: (d*sc)*q - dmin*m
      const uint4 h = lds16(raw + lane * 16);
      const uint4 q0 = lds16(raw + 512 + lane * 16), q1 = lds16(raw + 1024 + lane * 16);
      const float d = gb_half_to_float((uint16_t)(h.x & 0xFFFF)), dmin = gb_half_to_float((uint16_t)(h.x >> 16));
      uint8_t s[12];
#pragma unroll
      for (int i = 0; i < 12; i++) s[i] = byte_of(h, 4 + i);
      uint8_t m0, m1;
      const uint8_t sc0 = gb_q4k_scale(s, 2 * kc, &m0), sc1 = gb_q4k_scale(s, 2 * kc + 1, &m1);
      const float ds0 = __fmul_rn(d, (float)sc0), dm0 = __fmul_rn(dmin, (float)m0);
      const float ds1 = __fmul_rn(d, (float)sc1), dm1 = __fmul_rn(dmin, (float)m1);
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const bool hi = c >= 4;
        const int b0 = (c & 3) * 8;
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int bi = b0 + e;
          const uint8_t q = bi < 16 ? byte_of(q0, bi) : byte_of(q1, bi - 16);
          const int nib = hi ? (q >> 4) : (q & 0xF);
          v[e] = __fsub_rn(__fmul_rn(hi ? ds1 : ds0, (float)nib), hi ? dm1 : dm0);
        }
        put(c, v);
      }
      break;
    }
    case GB_T_Q4_0: {  // quant/quant.go:56-65: d*(q-8)
      const uint4 dd = lds16(raw + lane * 16);
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const int k = 2 * kc + b;
        const float d = gb_half_to_float((uint16_t)(byte_of(dd, 2 * k) | byte_of(dd, 2 * k + 1) << 8));
        const uint4 q = lds16(raw + 512 * (1 + b) + lane * 16);
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          const bool hi = cc >= 2;
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const uint8_t qb = byte_of(q, (cc & 1) * 8 + e);
            const int nib = hi ? (qb >> 4) : (qb & 0xF);
            v[e] = __fmul_rn(d, __fsub_rn((float)nib, 8.f));
          }
          put(4 * b + cc, v);
        }
      }
      break;
    }
    case GB_T_Q8_0: {  // quant/quant.go:44-55: d*q
      const uint4 dd = lds16(raw + lane * 16);
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const int k = 2 * kc + b;
        const float d = gb_half_to_float((uint16_t)(byte_of(dd, 2 * k) | byte_of(dd, 2 * k + 1) << 8));
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const uint4 q = lds16(raw + 512 * (1 + 2 * b + u) + lane * 16);
#pragma unroll
          for (int hlf = 0; hlf < 2; hlf++) {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = __fmul_rn(d, (float)(int8_t)byte_of(q, hlf * 8 + e));
            put(4 * b + 2 * u + hlf, v);
          }
        }
      }
      break;
    }
    case GB_T_Q6_K: {  // quant/quant.go:114-132: d*sc*(q-32)
      const uint8_t *ql = raw, *qh = raw + 2048, *sc = raw + 3072, *dp = raw + 3584;
      const int c = kc >> 1, q0 = (kc & 1) * 2;
      const float d = gb_half_to_float(*(const uint16_t *)(dp + lane * 2));
      const uint4 s4 = lds16(sc + lane * 16);
#pragma unroll
      for (int oc = 0; oc < 8; oc++) {
        const int quarter = q0 + (oc >> 2), l0 = (oc & 3) * 8;
        const int qlb = l0 + ((quarter & 1) ? 32 : 0);  // ql byte within the chunk's 64
        const uint4 L = lds16(ql + (qlb >> 4) * 512 + lane * 16);
        const uint4 H = lds16(qh + (l0 >> 4) * 512 + lane * 16);
        const int scv = (int8_t)byte_of(s4, c * 8 + 2 * quarter + (l0 >> 4));
        const float dsc = __fmul_rn(d, (float)scv);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const uint8_t lb = byte_of(L, (qlb & 15) + e), hb = byte_of(H, (l0 & 15) + e);
          const int lo = quarter >= 2 ? (lb >> 4) : (lb & 0xF);
          const int q = lo | (((hb >> (2 * quarter)) & 3) << 4);
          v[e] = __fmul_rn(dsc, (float)(q - 32));
        }
        put(oc, v);
      }
      break;
    }
    case GB_T_F16:
#pragma unroll
      for (int c2 = 0; c2 < 8; c2++) *(uint4 *)(row + ((c2 ^ sw) << 4)) = lds16(raw + c2 * 512 + lane * 16);
      break;
    case GB_T_BF16:
#pragma unroll
      for (int c2 = 0; c2 < 8; c2++) {
        const uint4 u = lds16(raw + c2 * 512 + lane * 16);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          v[2 * i] = __uint_as_float(w[i] << 16);
          v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
        put(c2, v);
      }
      break;
    case GB_T_F32:
#pragma unroll
      for (int c2 = 0; c2 < 8; c2++) {
        const uint4 a = lds16(raw + (2 * c2) * 512 + lane * 16), b = lds16(raw + (2 * c2 + 1) * 512 + lane * 16);
        v[0] = __uint_as_float(a.x), v[1] = __uint_as_float(a.y), v[2] = __uint_as_float(a.z), v[3] = __uint_as_float(a.w);
        v[4] = __uint_as_float(b.x), v[5] = __uint_as_float(b.y), v[6] = __uint_as_float(b.z), v[7] = __uint_as_float(b.w);
        put(c2, v);
      }
      break;
    default: {
#pragma unroll
      for (int c2 = 0; c2 < 8; c2++) *(uint4 *)(row + ((c2 ^ sw) << 4)) = make_uint4(0, 0, 0, 0);
    }
  }
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
  int nstage;
  int raw_tile;           // raw bytes per tile per stage (max over the two types)
  unsigned *err;
};

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

// BN: weight rows of the CTA (128, or 256 for gate/up pairs); NDQ = BN/32
// dequant warps (one 32-row tile each), then the producer warp, then the
// MMA warp.
template <int BN, int EPI>
__global__ void __launch_bounds__((BN / 32 + 2) * 32, 1)
    gemm_tc_kernel(const TcArgs g, const __grid_constant__ CUtensorMap tmap_a) {
  constexpr int NDQ = BN / 32;
  constexpr int BBytes = BN * 128;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kMaxStagesTC], bfull[kMaxStagesTC], empty[kMaxStagesTC], accf;
  __shared__ uint32_t tmem_base;
  __shared__ int bad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = g.nstage;
  const int nk = g.nsb * 4;                 // K stages
  const int m0 = blockIdx.y * kBM;          // first token row
  const int tile0 = blockIdx.x * 4;         // first weight tile (of each half for pairs)
  // [NS] A tiles | [NS] B tiles (1024-aligned) | [NS][NDQ] raw stage regions
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *A0 = base, *B0 = base + (size_t)NS * kABytes, *R0 = B0 + (size_t)NS * BBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      gb_mbar_init(&full[s], 1);
      gb_mbar_init(&bfull[s], NDQ * 32);
      gb_mbar_init(&empty[s], 1);
    }
    gb_mbar_init(&accf, 1);
    bad = 0;
    gb_mbar_fence_init();
  }
  if (warp == NDQ + 1) {
    tmem_alloc(&tmem_base, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == NDQ) {
    // producer: activation tile by TMA, the weight tiles' raw stage bytes by bulk copies
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < nk; k++) {
        const int s = k % NS;
        if (k >= NS && !gb_mbar_wait(&empty[s], ((k / NS) - 1) & 1)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        const int sb = k >> 2, kc = k & 3;
        uint32_t bytes = kABytes;
        for (int j = 0; j < NDQ; j++) {
          const int up = g.pair && j >= 4, tile = tile0 + (g.pair ? (j & 3) : j);
          if (tile >= g.ntiles) continue;
          int typ;
          (void)sb_block(g, tile, sb, up, typ);
          bytes += (uint32_t)stage_raw_bytes(typ);
        }
        gb_mbar_expect_tx(&full[s], bytes);
        tma_load_2d(A0 + (size_t)s * kABytes, &tmap_a, k * kBK, m0, &full[s]);
        for (int j = 0; j < NDQ; j++) {
          const int up = g.pair && j >= 4, tile = tile0 + (g.pair ? (j & 3) : j);
          if (tile >= g.ntiles) continue;
          int typ;
          const uint8_t *src = sb_block(g, tile, sb, up, typ);
          Piece pc[4];
          const int np = stage_pieces(typ, kc, pc);
          uint8_t *dst = R0 + ((size_t)s * NDQ + j) * g.raw_tile;
          for (int i = 0; i < np; i++) {
            gb_bulk_g2s(dst, src + pc[i].off, (uint32_t)pc[i].len, &full[s]);
            dst += pc[i].len;
          }
        }
        issued = k + 1;
      }
      // copies still in flight land (bounded) before the CTA exits
      for (int j = issued > NS ? issued - NS : 0; j < issued; j++) (void)gb_mbar_wait(&full[j % NS], (j / NS) & 1);
    }
  } else if (warp == NDQ + 1) {
    // MMA issue: one thread
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, BN);
      for (int k = 0; k < nk; k++) {
        const int s = k % NS;
        const uint32_t ph = (k / NS) & 1;
        if (!gb_mbar_wait(&full[s], ph) || !gb_mbar_wait(&bfull[s], ph)) {
          bad = 1;
          if (g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint64_t ad = sdesc_sw128(gb_smem_u32(A0 + (size_t)s * kABytes));
        const uint64_t bd = sdesc_sw128(gb_smem_u32(B0 + (size_t)s * BBytes));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++)  // K = 16 per instruction: +32 bytes in the swizzled row
          mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (k | kk) != 0);
        mma_commit(&empty[s]);  // the slot is free once these MMAs have read it
      }
      mma_commit(&accf);  // all issued MMAs done (also after an early stop)
    }
  } else {
    // dequant warps: warp j decodes tile j of the CTA, one row per lane
    const int j = warp;
    const int up = g.pair && j >= 4, tile = tile0 + (g.pair ? (j & 3) : j);
    const bool valid = tile < g.ntiles;
    for (int k = 0; k < nk; k++) {
      const int s = k % NS;
      const uint32_t ph = (k / NS) & 1;
      if (!gb_mbar_wait(&full[s], ph)) {
        if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
        bad = 1;
        break;
      }
      int typ = -1;  // a tile past the matrix decodes to zeros
      if (valid) (void)sb_block(g, tile, k >> 2, up, typ);
      dequant_stage(typ, k & 3, R0 + ((size_t)s * NDQ + j) * g.raw_tile, lane, B0 + (size_t)s * BBytes, j * 32 + lane);
      gb_fence_proxy_async();
      gb_mbar_arrive(&bfull[s]);
    }
    // epilogue: accumulators -> registers -> global
    const bool ok = gb_mbar_wait(&accf, 0);
    tc_fence_after();
    if (!ok) {
      if (lane == 0 && g.err) atomicOr(g.err, GB_DEVERR_TIMEOUT);
    } else if (!bad) {
      const int quarter = warp & 3;  // tcgen05.ld reaches TMEM lanes 32*(warp%4)..+31
      const int m = m0 + quarter * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
      if constexpr (EPI == GB_EPI_SWIGLU) {
        // warps 0-3 take columns 0..63 of gate and up, warps 4-7 columns 64..127
        const int c0 = (warp >> 2) * 64;
        for (int cc = c0; cc < c0 + 64; cc += 16) {
          float gv[16], uv[16];
          tmem_ld16(trow + cc, gv);
          tmem_ld16(trow + 128 + cc, uv);
          const int n = tile0 * 32 + cc;
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
        for (int cc = 0; cc < BN; cc += 16) {
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
            for (int i = 0; i < 16 && n + i < g.rows; i++) dst[i] = EPI == GB_EPI_RESID ? dst[i] + v[i] : v[i];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == NDQ + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
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
__global__ void rmsnorm_rows_f16_kernel(const float *x, const float *w, int n, float eps, __half *out) {
  const float *xr = x + (size_t)blockIdx.x * n;
  __half *o = out + (size_t)blockIdx.x * n;
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
  const float inv = (float)(1.0 / sqrt(red[0] / (double)n + (double)eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __float2half_rn(__fmul_rn(__fmul_rn(xr[i], inv), w[i]));
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
  for (int i = threadIdx.x; i < pairs + kv_rows; i += blockDim.x) {
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

}  // namespace

// ---- launchers ------------------------------------------------------------------

int gb_tmap_f16_rows(const void *base, int rows, int cols, CUtensorMap *map) {
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
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return gb_fail(GB_ERR_CUDA, "gpu: prefill: tensor map encode failed (%d)", (int)r);
  return GB_OK;
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
  g.raw_tile = (std::max(stage_raw_bytes(a.type_a), stage_raw_bytes(a.type_b)) + 127) & ~127;
  const int BN = g.pair ? 256 : 128, NDQ = BN / 32;
  const size_t stage = (size_t)kABytes + (size_t)BN * 128 + (size_t)NDQ * g.raw_tile;
  const size_t budget = 227 * 1024 - 1024 - 256;  // dynamic smem minus the alignment slack and statics
  int ns = (int)(budget / stage);
  if (ns > kMaxStagesTC) ns = kMaxStagesTC;
  if (ns < 2) return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: stage of %zu bytes does not fit", stage);
  g.nstage = ns;
  const size_t smem = (size_t)ns * stage + 1024;
  dim3 grid((unsigned)((a.rows + 127) / 128), (unsigned)((a.T + kBM - 1) / kBM));
  if (g.pair) grid.x = (unsigned)((a.rows + 127) / 128);  // rows = FFN rows of one half
  const dim3 block((unsigned)((NDQ + 2) * 32));
  void (*kern)(TcArgs, CUtensorMap) = nullptr;
  switch (a.epi) {
    case GB_EPI_PLAIN: kern = gemm_tc_kernel<128, GB_EPI_PLAIN>; break;
    case GB_EPI_RESID: kern = gemm_tc_kernel<128, GB_EPI_RESID>; break;
    case GB_EPI_SWIGLU: kern = gemm_tc_kernel<256, GB_EPI_SWIGLU>; break;
    default: return gb_fail(GB_ERR_UNSUPPORTED, "gpu: prefill: epilogue %d", a.epi);
  }
  GB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "gpu: prefill GEMM");
  kern<<<grid, block, smem, st>>>(g, a.tmap_a);
  GB_CUDA(cudaGetLastError(), "gpu: prefill GEMM");
  return GB_OK;
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
  rmsnorm_rows_f16_kernel<<<rows, 256, 0, st>>>(x, w, n, eps, out);
  GB_CUDA(cudaGetLastError(), "gpu: prefill RMSNorm");
  return GB_OK;
}

int gb_rope_kv_launch(const float *qkv, int T, int q_rows, int kv_rows, int hd, const double *rope_cs, int pos0,
                      int max_len, int kv_f16, float *q_out, void *kcache, void *vcache, cudaStream_t st) {
  rope_kv_kernel<<<T, 256, 0, st>>>(qkv, q_rows + 2 * kv_rows, q_rows, kv_rows, hd, rope_cs, pos0, max_len, kv_f16,
                                    q_out, kcache, vcache);
  GB_CUDA(cudaGetLastError(), "gpu: prefill RoPE");
  return GB_OK;
}

int gb_attn_prefill_launch(const float *q, int T, int pos0, int n_heads, int n_kv, int hd, const void *kcache,
                           const void *vcache, int kv_f16, int max_len, __half *out, cudaStream_t st) {
  const int G = n_heads / n_kv;
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
