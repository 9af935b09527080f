// layout.cuh — device layouts of the quantised weight matrices.
//
// A row is cut into 2048-value groups:
//   Q4_K  group = 8 GGUF blocks of 144 B, unchanged         (1152 B)
//   Q6_K  group = 8 x (ql 128 | qh 64 | scales 16) = 1664 B, then the 8 fp16
//         super-block scales                               (1680 B)
//   Q8_0  group = 64 x qs[32] = 2048 B, then the 64 fp16 scales (2176 B)
// A shorter last group (rows not a multiple of 2048 values) keeps the same
// order and is padded to 16 bytes; `row_bytes_dev` is the sum of a row's
// group pieces.
//
// Matrices are stored tile-major: 8 consecutive rows form a tile, and inside
// a tile the pieces are ordered group first, row second:
//   tile i = [group 0: row 8i .. 8i+7][group 1: row 8i .. 8i+7] ...
// so one (tile, group) stage — the unit the streaming GEMV moves with one
// bulk copy — is a single contiguous, 16-byte aligned range of
// 8 * piece bytes. A matrix whose row count is not a multiple of 8 is padded
// with zero rows to a whole tile. The repack is a bijection of the GGUF bytes,
// so every integer the kernels form is the one the reference forms.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define FB_HD __host__ __device__ __forceinline__
#else
#define FB_HD inline
#endif

namespace fb {

constexpr int kGroupValues = 2048;
constexpr int kTileRows = 8;

FB_HD int blocks_per_group(int type) { return type == 8 ? 64 : 8; }   // Q8_0 : K-quants
FB_HD int quant_bytes(int type) { return type == 8 ? 32 : (type == 14 ? 208 : 144); }
FB_HD bool has_dtab(int type) { return type == 8 || type == 14; }
FB_HD bool is_tiled(int type) { return type == 8 || type == 12 || type == 14; }

// bytes of a group holding gb blocks (padded to 16)
FB_HD size_t group_bytes(int type, int gb) {
    size_t b = (size_t)gb * quant_bytes(type) + (has_dtab(type) ? (size_t)gb * 2 : 0);
    return (b + 15) / 16 * 16;
}

// blocks in a row of n values
FB_HD int row_blocks(int type, int n) { return type == 8 ? n / 32 : n / 256; }

// offset of group gi inside a row's sequence of pieces (all earlier groups full)
FB_HD size_t group_offset(int type, int gi) { return (size_t)gi * group_bytes(type, blocks_per_group(type)); }

// number of blocks in group gi of a row with nb blocks
FB_HD int group_blocks(int type, int nb, int gi) {
    const int bpg = blocks_per_group(type);
    const int r = nb - gi * bpg;
    return r < bpg ? r : bpg;
}

FB_HD int row_groups(int type, int n) {
    const int nb = row_blocks(type, n), bpg = blocks_per_group(type);
    return (nb + bpg - 1) / bpg;
}

FB_HD size_t row_bytes_dev(int type, int n) {
    const int nb = row_blocks(type, n), bpg = blocks_per_group(type);
    const int full = nb / bpg, rem = nb % bpg;
    return (size_t)full * group_bytes(type, bpg) + (rem ? group_bytes(type, rem) : 0);
}

// bytes of a whole matrix of `rows` rows (whole tiles)
FB_HD size_t tiled_matrix_bytes(int type, int n, int rows) {
    return (size_t)((rows + kTileRows - 1) / kTileRows) * kTileRows * row_bytes_dev(type, n);
}

// byte offset of row `row`'s group gi inside a tiled matrix
FB_HD size_t piece_offset(int type, int n, int row, int gi) {
    const int nb = row_blocks(type, n);
    const size_t rb = row_bytes_dev(type, n);
    return (size_t)(row / kTileRows) * kTileRows * rb + kTileRows * group_offset(type, gi) +
           (size_t)(row % kTileRows) * group_bytes(type, group_blocks(type, nb, gi));
}

// quant bytes of block b of a row (Q4_K: the whole 144-byte block)
FB_HD size_t block_offset_tm(int type, int n, int row, int b) {
    const int bpg = blocks_per_group(type);
    return piece_offset(type, n, row, b / bpg) + (size_t)(b % bpg) * quant_bytes(type);
}

// fp16 scale of block b of a row (Q6_K / Q8_0)
FB_HD size_t dscale_offset_tm(int type, int n, int row, int b) {
    const int bpg = blocks_per_group(type), gi = b / bpg, nb = row_blocks(type, n);
    return piece_offset(type, n, row, gi) + (size_t)group_blocks(type, nb, gi) * quant_bytes(type) +
           2 * (size_t)(b % bpg);
}

}  // namespace fb
