// gb_formats.h -- ggml block formats (gguf/types.go:47-81) and the B200
// tiled weight layout, shared by host and device code.
//
// Tiled layout of a quantized [rows][cols] matrix (cols a multiple of 256):
// rows are grouped into tiles of 32 (the last tile zero-padded). For every
// tile and every 256-element super-block `sb` of the row, the 32 rows'
// bytes form one contiguous "sb-block" of 16-byte units, unit-major and
// row(lane)-minor: unit u of the row in lane l lives at u*512 + l*16. A warp
// therefore reads each unit of 32 rows as one 512-byte coalesced access,
// and one 1-D TMA bulk copy moves a whole sb-block into shared memory.
//   Q4_K: 9 units = the raw 144-byte block cut in 16-byte pieces
//         (unit 0 = d, dmin, 12 scale bytes; units 1..8 = the 128 quant bytes).
//   Q5_K: 11 units = the raw 176-byte block cut in 16-byte pieces (unit 0 =
//         d, dmin, 12 scale bytes; units 1..2 = the 32 fifth-bit bytes qh;
//         units 3..10 = the 128 low-nibble bytes qs).
//   Q6_K: 13 units = raw bytes [0,208) (ql 8, qh 4, scales 1), then the
//         32 rows' 2-byte d at 13*512 + l*2 (sb-block 6720 bytes = 32*210).
//   Q4_0: the 8 raw 18-byte blocks of the super-block are regrouped:
//         unit 0 = the eight binary16 d, unit 1+k = the 16 quant bytes of
//         block k (sb-block 4608 bytes = 32*144).
//   Q8_0: the 8 raw 34-byte blocks likewise: unit 0 = the eight binary16 d,
//         units 1+2k, 2+2k = the 32 int8 quants of block k (17 units,
//         sb-block 8704 bytes = 32*272).
//   F16 / BF16 / F32: the row's 256 elements in order, 8 or 4 per unit
//         (32 or 64 units, sb-block 16384 or 32768 bytes).
// The tiled buffer holds exactly the raw bytes (plus row padding), so a
// decode step reads the algorithmic byte count.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define GB_HD __host__ __device__ __forceinline__
#else
#define GB_HD inline
#endif

// Error flags a kernel can raise in the model's device status word.
#define GB_DEVERR_POS 1u      // position outside the KV cache
#define GB_DEVERR_TOKEN 2u    // token outside the vocabulary
#define GB_DEVERR_TIMEOUT 4u  // a bounded mbarrier wait ran out

enum {
  GB_T_F32 = 0, GB_T_F16 = 1, GB_T_Q4_0 = 2, GB_T_Q8_0 = 8, GB_T_Q4_K = 12, GB_T_Q5_K = 13, GB_T_Q6_K = 14,
  GB_T_BF16 = 30
};

// gguf/types.go:47-57 (the subset with kernels here; 0 = unsupported).
GB_HD int gb_block_size(int t) {
  switch (t) {
    case GB_T_F32: case GB_T_F16: case GB_T_BF16: return 1;
    case GB_T_Q4_0: case GB_T_Q8_0: return 32;
    case GB_T_Q4_K: case GB_T_Q5_K: case GB_T_Q6_K: return 256;
  }
  return 0;
}
GB_HD int gb_type_size(int t) {
  switch (t) {
    case GB_T_F32: return 4;
    case GB_T_F16: case GB_T_BF16: return 2;
    case GB_T_Q4_0: return 18;
    case GB_T_Q8_0: return 34;
    case GB_T_Q4_K: return 144;
    case GB_T_Q5_K: return 176;
    case GB_T_Q6_K: return 210;
  }
  return 0;
}
// gguf/types.go:81 RowBytes.
GB_HD int64_t gb_row_bytes(int t, int64_t n) {
  int bs = gb_block_size(t);
  return bs ? n / bs * gb_type_size(t) : 0;
}

// Unquantized weight matrices (model.uploadLinear, model/model.go:86-96: F16
// and F32; BF16 added, as the embedding accepts any known type).
GB_HD bool gb_float_type(int t) { return t == GB_T_F16 || t == GB_T_BF16 || t == GB_T_F32; }
GB_HD bool gb_tiled_type(int t) {
  return t == GB_T_Q4_0 || t == GB_T_Q8_0 || t == GB_T_Q4_K || t == GB_T_Q5_K || t == GB_T_Q6_K || gb_float_type(t);
}
GB_HD int gb_tiled_units(int t) {
  return t == GB_T_Q6_K ? 13 : t == GB_T_Q5_K ? 11 : t == GB_T_Q8_0 ? 17 : (t == GB_T_F16 || t == GB_T_BF16) ? 32 : t == GB_T_F32 ? 64 : 9;
}
GB_HD int gb_tiled_sb_bytes(int t) {
  return t == GB_T_Q6_K ? 6720
         : t == GB_T_Q5_K ? 5632
         : t == GB_T_Q8_0 ? 8704
         : (t == GB_T_F16 || t == GB_T_BF16) ? 16384
         : t == GB_T_F32 ? 32768
                          : 4608;
}

// Where raw byte `b` (0 <= b < 32*typesize/... of one super-block of a row)
// lives inside the sb-block, for lane `lane`.
GB_HD int gb_tiled_offset(int t, int lane, int b) {
  if (t == GB_T_Q4_0) {
    int k = b / 18, w = b % 18;
    if (w < 2) return lane * 16 + 2 * k + w;
    return (1 + k) * 512 + lane * 16 + (w - 2);
  }
  if (t == GB_T_Q8_0) {
    int k = b / 34, w = b % 34;
    if (w < 2) return lane * 16 + 2 * k + w;
    int q = w - 2;
    return (1 + 2 * k + q / 16) * 512 + lane * 16 + (q & 15);
  }
  if (t == GB_T_Q6_K && b >= 208) return 13 * 512 + lane * 2 + (b - 208);
  return (b >> 4) * 512 + lane * 16 + (b & 15);
}
// Raw bytes per super-block of one row (256 elements).
GB_HD int gb_sb_raw_bytes(int t) {
  return t == GB_T_Q6_K ? 210 : t == GB_T_Q5_K ? 176 : t == GB_T_Q8_0 ? 272 : (t == GB_T_F16 || t == GB_T_BF16) ? 512 : t == GB_T_F32 ? 1024 : 144;
}
