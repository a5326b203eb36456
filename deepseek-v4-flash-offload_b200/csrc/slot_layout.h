// Byte layout of the packed expert slot, shared by the host packer and the
// device kernels.
//
// Both weight matrices are stored as "row-tile pairs": 256 rows x 128 K
// elements = one contiguous 16 KiB block of packed E2M1 (64 B per row), so a
// single TMA box brings both 128-row operand tiles of a GEMM step:
//   * w13: pair p = (w1 rows 128p..128p+127, then w3 rows 128p..128p+127),
//     the gate and up rows that the same SwiGLU epilogue needs;
//   * w2 : pair p = rows 256p..256p+255 (two consecutive 128-row tiles).
// Blocks are ordered (pair, k-tile).  The E8M0 scales follow the same order:
// per (pair, k-tile) 1 KiB = two 512-byte atoms, one per 128-row half, row r
// of a half at (r%32)*16 + (r/32)*4, 32-element block kb%4 in the low bits;
// the order the tensor cores read after a tcgen05.cp 32x128b.warpx4.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define DSV4_HD __host__ __device__ __forceinline__
#else
#define DSV4_HD inline
#endif

namespace dsv4 {

// Paired-matrix row of w1 row r (which = 0) or w3 row r (which = 1).
DSV4_HD int64_t w13_pair_row(int64_t r, int which) { return (r / 128) * 256 + (int64_t)which * 128 + r % 128; }

// Byte holding elements (k0, k0+1) of paired-matrix row R (k0 even), K = row length.
DSV4_HD int64_t w_pair_offset(int64_t R, int64_t k0, int64_t K) {
  return ((R / 256) * (K / 128) + k0 / 128) * 16384 + (R % 256) * 64 + (k0 % 128) / 2;
}

// Byte of the scale of (paired-matrix row R, 32-element block kb).
DSV4_HD int64_t sf_pair_offset(int64_t R, int64_t kb, int64_t K) {
  const int64_t r = R % 128;
  return ((R / 256) * (K / 128) + kb / 4) * 1024 + ((R % 256) / 128) * 512 + (r % 32) * 16 + (r / 32) * 4 + kb % 4;
}

// FP8 (E4M3) slot of the shared expert: the same pairs, blocks and scale
// atoms, one byte per element, so a block is 256 rows x 128 B = 32 KiB and
// lands in shared memory exactly like an expanded E2M1 block.
DSV4_HD int64_t w8_pair_offset(int64_t R, int64_t k, int64_t K) {
  return ((R / 256) * (K / 128) + k / 128) * 32768 + (R % 256) * 128 + k % 128;
}

}  // namespace dsv4
