// gb_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// binary16 helpers, bit-exact ggml block decoders, the u8 x s8 dot product,
// 1-D TMA bulk copies with mbarrier completion and bounded waits, warp
// reductions, and the "limb pack" of an activation vector.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "gb_formats.h"

#define GB_DEV __device__ __forceinline__

// Iteration limit of every mbarrier wait: each try_wait may suspend for a
// hardware-defined time slice, so this bounds a wait at well under a second.
#define GB_WAIT_LIMIT (1u << 20)

GB_DEV float gb_half_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }
GB_DEV uint16_t gb_float_to_half_rn(float f) { return __half_as_ushort(__float2half_rn(f)); }

// ---- bit-exact decoders (the arithmetic of quant.Dequantize, quant/quant.go:27-132).
// __fmul_rn/__fsub_rn forbid FMA contraction so each f32 operation rounds
// on its own, as in the Go code.

GB_DEV uint8_t gb_q4k_scale(const uint8_t *s, int j, uint8_t *m) {
  // quant.ScaleMinQ4K, quant/quant.go:90
  if (j < 4) {
    *m = s[j + 4] & 63;
    return s[j] & 63;
  }
  *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  return (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
}

// Element e of one raw block (blk points at the block's bytes).
GB_DEV float gb_dequant_elem(int typ, const uint8_t *blk, int e) {
  switch (typ) {
    case GB_T_Q4_0: {  // quant/quant.go:56-65: d*(q-8)
      float d = gb_half_to_float((uint16_t)(blk[0] | blk[1] << 8));
      uint8_t q = blk[2 + (e & 15)];
      int nib = e < 16 ? (q & 0xF) : (q >> 4);
      return __fmul_rn(d, __fsub_rn((float)nib, 8.f));
    }
    case GB_T_Q8_0: {
      float d = gb_half_to_float((uint16_t)(blk[0] | blk[1] << 8));
      return __fmul_rn(d, (float)(int8_t)blk[2 + e]);
    }
    case GB_T_Q4_K: {  // quant/quant.go:97-112: (d*sc)*q - dmin*m
      float d = gb_half_to_float((uint16_t)(blk[0] | blk[1] << 8));
      float dmin = gb_half_to_float((uint16_t)(blk[2] | blk[3] << 8));
      int chunk = e >> 6, w = e & 63, l = w & 31, hi = w >> 5;
      uint8_t m;
      uint8_t sc = gb_q4k_scale(blk + 4, 2 * chunk + hi, &m);
      uint8_t q = blk[16 + chunk * 32 + l];
      int nib = hi ? (q >> 4) : (q & 0xF);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)nib), __fmul_rn(dmin, (float)m));
    }
    case GB_T_Q5_K: {  // ggml block_q5_K (not decoded by the reference): (d*sc)*q - dmin*m, q 5 bits
      float d = gb_half_to_float((uint16_t)(blk[0] | blk[1] << 8));
      float dmin = gb_half_to_float((uint16_t)(blk[2] | blk[3] << 8));
      int chunk = e >> 6, w = e & 63, l = w & 31, hi = w >> 5;
      uint8_t m;
      uint8_t sc = gb_q4k_scale(blk + 4, 2 * chunk + hi, &m);
      uint8_t q = blk[48 + chunk * 32 + l];
      int v = (hi ? (q >> 4) : (q & 0xF)) | (((blk[16 + l] >> (2 * chunk + hi)) & 1) << 4);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)v), __fmul_rn(dmin, (float)m));
    }
    case GB_T_Q6_K: {  // quant/quant.go:114-132: d*sc*(q-32)
      int chunk = e >> 7, w = e & 127, quarter = w >> 5, l = w & 31, is = l >> 4;
      const uint8_t *l0 = blk + chunk * 64, *h0 = blk + 128 + chunk * 32;
      const int8_t *s0 = (const int8_t *)(blk + 192 + chunk * 8);
      float d = gb_half_to_float((uint16_t)(blk[208] | blk[209] << 8));
      int q, sc;
      switch (quarter) {
        case 0: q = (l0[l] & 0xF) | ((h0[l] & 3) << 4); sc = s0[is]; break;
        case 1: q = (l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4); sc = s0[is + 2]; break;
        case 2: q = (l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4); sc = s0[is + 4]; break;
        default: q = (l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4); sc = s0[is + 6]; break;
      }
      return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));
    }
    case GB_T_F16: return gb_half_to_float((uint16_t)(blk[2 * e] | blk[2 * e + 1] << 8));
    case GB_T_BF16: return __uint_as_float((uint32_t)(blk[2 * e] | blk[2 * e + 1] << 8) << 16);
    case GB_T_F32: {
      uint32_t b = (uint32_t)blk[4 * e] | (uint32_t)blk[4 * e + 1] << 8 |
                   (uint32_t)blk[4 * e + 2] << 16 | (uint32_t)blk[4 * e + 3] << 24;
      return __uint_as_float(b);
    }
  }
  return 0.f;
}

// ---- integer dot product: 4 unsigned bytes x 4 signed bytes + c.
GB_DEV int gb_dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 4 signed bytes x 4 signed bytes + c.
GB_DEV int gb_dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---- warp reductions
GB_DEV float gb_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
GB_DEV float gb_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- 1-D TMA bulk copies and mbarriers (sm_90+; used here for sm_100a)
GB_DEV uint32_t gb_smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

GB_DEV void gb_mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(gb_smem_u32(bar)), "r"(count)
               : "memory");
}
GB_DEV void gb_mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
GB_DEV void gb_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Order this thread's later async-proxy (TMA) reads of global memory after
// what the generic proxy wrote there (the preceding kernel's stores).
GB_DEV void gb_fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
GB_DEV void gb_mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(gb_smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Global -> shared bulk copy completing on bar. dst, src and bytes must be
// multiples of 16.
GB_DEV void gb_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          gb_smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(gb_smem_u32(bar))
      : "memory");
}
// Tiled 4-D TMA load of one box of the tensor map `tmap` (a __grid_constant__
// kernel parameter) at coordinates (c0 innermost .. c3) into dst, completing
// on bar. c0 * element size must be a multiple of 16 bytes; no multicast.
GB_DEV void gb_tma_load_4d(void *dst, const void *tmap, int c0, int c1, int c2, int c3, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(gb_smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(gb_smem_u32(bar))
      : "memory");
}
GB_DEV void gb_mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(gb_smem_u32(bar)) : "memory");
}
GB_DEV bool gb_mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(gb_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity; false on timeout.
GB_DEV bool gb_mbar_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < GB_WAIT_LIMIT; i++)
    if (gb_mbar_try_wait(bar, parity)) return true;
  return false;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// let the next grid start its prologue early. Both are no-ops when the
// launch did not enable programmatic serialization.
GB_DEV void gb_grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
GB_DEV void gb_grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// System-scope flag accesses for peer (NVLink) signalling.
GB_DEV unsigned gb_ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
GB_DEV void gb_st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 64-bit accesses that other GPUs read over NVLink while this one writes them
// (aligned 64-bit scalar accesses are single-copy atomic).
GB_DEV void gb_st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
GB_DEV unsigned long long gb_ld_relaxed_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Streaming 16-byte global load that does not allocate in L1.
GB_DEV uint4 gb_ld_stream16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---- the limb form of an activation block ---------------------------------
// A GEMV stages each 256-element super-block of its input as a scale
// s = max|x|/127 and three signed-byte limbs per element with
//   x ~= s * (a + b/254 + c/254^2),  a,b,c in [-127,127],
// which represents x to within s/2/254^2 (about 6e-8 of the block's largest
// magnitude, the float32 rounding level). Quantized matrix-vector products
// then run on dp4a with exact int32 sums (gb_gemv.cu).

// ---- mma.sync m16n8k16 (f16 in, f32 accumulate) and ldmatrix, shared by the
// attention kernels
GB_DEV uint32_t h2pack(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// fp16 rounding of (x0, x1) and of the residues
GB_DEV void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = h2pack(h0, h1);
  lo = h2pack(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
}
GB_DEV void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
GB_DEV void ldsm_x4(uint32_t r[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(gb_smem_u32(p)));
}
GB_DEV void ldsm_x4_t(uint32_t r[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(gb_smem_u32(p)));
}
